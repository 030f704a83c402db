// api.cu — host side of the orchkv data plane (orchkv_* C ABI).
//
// The reference keeps one global system (src/api/orchkv_api.cu:20-30) with a
// cudaMalloc'd GPU slab pool, a pinned DRAM slab pool, host LIFO free stacks
// and per-request host block vectors, and moves each slab with its own
// cudaMemcpyAsync + stream sync.  Here the same global system keeps pools,
// free stacks, block locations and request block tables in GPU-visible memory;
// every state change is made by a kernel on one stream, so per-block calls
// and batched calls observe one consistent state.  The DRAM pool is pinned
// and mapped, so migration kernels read and write it directly over the host
// link (fused gather+D2H and H2D+scatter).
#include <errno.h>
#include <fcntl.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>
#include <sys/uio.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <thread>
#include <unordered_set>

#include <map>
#include <mutex>
#include <vector>

#include "kernels.h"
#include "orchkv/orchkv_api.h"
#include "pool.h"
#include "tm_internal.h"

using namespace okv;

struct kv_request_ctx {
    uint64_t request_id;
    uint32_t L, H, mbph;
    size_t region_off;     // words into the block-table array
    size_t region_words;
    int fd = -1;           // storage-tier file (src/tiered_store/orchfs_tier.c:201-244)
    char path[256] = {0};
};

namespace {

constexpr uint32_t kStagedMin = 2048;        // batches this large may use the copy engine
constexpr size_t kChunkBytes = 256u << 20;   // staging ring slot size
constexpr int kRing = 3;
constexpr int kMaxChunks = 1024;
constexpr uint32_t kMaxRuns = 65536;         // DRAM runs per staged evict
constexpr size_t kCeMinRunBytes = 1u << 20;  // shorter DRAM runs are written zero-copy

struct Sys {
    std::recursive_mutex mu;
    bool inited = false;
    orchkv_config_t cfg;
    int device = 0;
    cudaStream_t own = nullptr, stream = nullptr;
    PoolDev p;
    char *dev_meta = nullptr;         // stacks, loc/state/flags, counters
    uint32_t *bt = nullptr;           // block-table array
    size_t bt_words = 0;
    std::map<size_t, size_t> free_regions;   // offset -> words
    uint32_t *scratch = nullptr;
    size_t scratch_words = 0;
    CompatResult *res = nullptr;      // pinned
    PoolCounters *h_ctr = nullptr;    // pinned
    char *stage = nullptr;            // device staging for pageable inputs
    size_t stage_cap = 0;
    uint32_t **regions_dev = nullptr; // device array of region pointers
    uint32_t **regions_host = nullptr;// pinned
    uint32_t regions_cap = 0;
    std::vector<uint32_t *> regions_last;
    tiered_manager_t *attached = nullptr;
    uint32_t active_requests = 0;
    // staged evict: device staging ring drained to the DRAM tier by the copy
    // engine on its own stream; per-chunk events time the pack kernels
    cudaStream_t copy = nullptr;
    char *ring = nullptr;             // ev_copied.size() slots of ring_slabs slabs
    uint32_t ring_slabs = 0;          // slabs per ring slot
    std::vector<cudaEvent_t> ev_copied;
    cudaEvent_t ev_pk[2 * kMaxChunks] = {};
    cudaEvent_t ev_up[2 * kMaxChunks] = {};       // around each unpack launch of a promote
    uint32_t last_unpacks = 0;
    unsigned long long last_unpack_bytes[kMaxChunks] = {};
    cudaEvent_t ev_mig[4] = {};
    cudaEvent_t ev_packed = nullptr;  // all of a swap's victims packed
    char *sort_mem = nullptr;         // SortScratch storage (evict, then promote)
    SortScratch ss, ss2;
    uint32_t *h_runs = nullptr;       // pinned: run_o then run_d (evict)
    uint32_t *h_runs2 = nullptr;      // pinned: run_o then run_d (promote)
    char *h_cold = nullptr;           // pinned, mapped: staging of batched cold evicts (2 halves)
    cudaEvent_t ev_cold[2] = {};      // each half gathered
    uint32_t *h_meta = nullptr;       // pinned
    // staged promote: copy-engine H2D on copy_in into its own ring, unpack
    // kernels on their own stream
    cudaStream_t copy_in = nullptr, unpack = nullptr;
    char *pring = nullptr;            // kRing slots of ring_slabs slabs
    cudaEvent_t ev_h2d[kMaxChunks] = {};
    cudaEvent_t ev_unpacked[kRing] = {};
    cudaEvent_t ev_in_done = nullptr;
    uint32_t *scratch2 = nullptr;     // the promote plan of a swap
    size_t scratch2_words = 0;
    uint32_t last_chunks = 0;
    int last_evict_staged = 0, last_promote_timed = 0;
    unsigned long long last_pack_bytes = 0;
    uint32_t last_runs = 0, last_ce_copies = 0, last_zc_slabs = 0;
    uint32_t last_p_runs = 0, last_p_ce_copies = 0, last_p_zc_slabs = 0;
    int last_swap_overlapped = 0;
    uint32_t last_swap_conflicts = 0;
    gpu_tier_t gsnap;
    dram_tier_t dsnap;
    orchfs_tier_t fsnap;
    std::vector<uint32_t> gsnap_stack, dsnap_stack;
    // storage tier
    char base_dir[256] = {0};
    uint64_t storage_writes = 0, storage_reads = 0;
    uint64_t storage_bytes_written = 0, storage_bytes_read = 0;
};

// mkdir -p (src/tiered_store/orchfs_tier.c:152-165)
void mkdir_p(const char *path)
{
    char tmp[256];
    snprintf(tmp, sizeof(tmp), "%s", path);
    for (char *q = tmp + 1; *q; q++) {
        if (*q == '/') {
            *q = '\0';
            mkdir(tmp, 0755);
            *q = '/';
        }
    }
    mkdir(tmp, 0755);
}

Sys g;

uint32_t pow2_at_least(uint64_t v)
{
    uint64_t c = 1;
    while (c < v) c <<= 1;
    return (uint32_t)c;
}

ReqDev req_dev(const kv_request_ctx *c)
{
    ReqDev r;
    r.region = g.bt + c->region_off;
    r.L = c->L;
    r.H = c->H;
    r.mbph = c->mbph;
    return r;
}

// Checked build: out-of-range indices met so far, folded in from the device
// words (which shutdown frees); {count, line, index, bound} of the first.
uint32_t g_check_tally[4] = {0, 0, 0, 0};

int fold_check_words()
{
    if (!kCheckedBuild || !g.p.chk) return ORCHKV_OK;
    uint32_t w[4];
    OKV_CUDA_TRY(cudaMemcpy(w, g.p.chk, sizeof(w), cudaMemcpyDeviceToHost));
    if (w[0] == 0) return ORCHKV_OK;
    if (g_check_tally[0] == 0) {
        fprintf(stderr, "[orchkv] checked build: %u index(es) out of range; first at "
                        "pool_kernels.cu:%u (index %u, bound %u)\n", w[0], w[1], w[2], w[3]);
        memcpy(g_check_tally + 1, w + 1, 3 * sizeof(uint32_t));
    }
    g_check_tally[0] += w[0];
    OKV_CUDA_TRY(cudaMemset(g.p.chk, 0, sizeof(w)));
    return ORCHKV_OK;
}

// ORCHKV_ERR_CUDA once a checked build met an index out of range (until
// orchkv_check_status resets the tally).
int check_words()
{
    const int rc = fold_check_words();
    if (rc) return rc;
    return g_check_tally[0] ? ORCHKV_ERR_CUDA : ORCHKV_OK;
}

int sync_result(int *rc_out)
{
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    if (rc_out) *rc_out = g.res->rc;
    return ORCHKV_OK;
}

// A caller pointer kernels can read in place: device, managed or mapped
// pinned memory.  nullptr for pageable host memory.
const char *direct_ptr(const void *ptr)
{
    cudaPointerAttributes a;
    cudaError_t e = cudaPointerGetAttributes(&a, ptr);
    if (e == cudaSuccess && (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged))
        return (const char *)ptr;
    if (e == cudaSuccess && a.type == cudaMemoryTypeHost && a.devicePointer)
        return (const char *)a.devicePointer;
    cudaGetLastError();   // clear a failed attribute query
    return nullptr;
}

// Resolve the K and V inputs of one call (`bytes` each): used in place when
// kernels can read them, else copied into the staging buffer.  The buffer is
// grown for both before either copy is queued, so a growth never strands a
// pointer handed out for the first.
int resolve_kv(const void *k, const void *v, size_t bytes, const char **kd, const char **vd)
{
    *kd = k ? direct_ptr(k) : nullptr;
    *vd = v ? direct_ptr(v) : nullptr;
    const bool stage_k = k && !*kd, stage_v = v && !*vd;
    const size_t need = (stage_k ? bytes : 0) + (stage_v ? bytes : 0);
    if (need == 0) return ORCHKV_OK;
    if (need > g.stage_cap) {
        size_t cap = g.stage_cap ? g.stage_cap : (1 << 20);
        while (cap < need) cap *= 2;
        OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));   // earlier copies may still read it
        cudaFree(g.stage);
        g.stage = nullptr;
        g.stage_cap = 0;
        OKV_CUDA_TRY(cudaMalloc((void **)&g.stage, cap));
        g.stage_cap = cap;
    }
    size_t off = 0;
    if (stage_k) {
        OKV_CUDA_TRY(cudaMemcpyAsync(g.stage, k, bytes, cudaMemcpyHostToDevice, g.stream));
        *kd = g.stage;
        off = bytes;
    }
    if (stage_v) {
        OKV_CUDA_TRY(cudaMemcpyAsync(g.stage + off, v, bytes, cudaMemcpyHostToDevice, g.stream));
        *vd = g.stage + off;
    }
    return ORCHKV_OK;
}

int upload_regions(kv_request_ctx_t *const *ctxs, uint32_t n, uint32_t *L, uint32_t *H,
                   uint32_t *mbph)
{
    if (!ctxs || n == 0) return ORCHKV_ERR_INVALID;
    for (uint32_t i = 0; i < n; i++) {
        if (!ctxs[i]) return ORCHKV_ERR_INVALID;
        if (ctxs[i]->L != ctxs[0]->L || ctxs[i]->H != ctxs[0]->H) return ORCHKV_ERR_INVALID;
    }
    *L = ctxs[0]->L;
    *H = ctxs[0]->H;
    *mbph = ctxs[0]->mbph;
    std::vector<uint32_t *> want(n);
    for (uint32_t i = 0; i < n; i++) want[i] = g.bt + ctxs[i]->region_off;
    if (want == g.regions_last) return ORCHKV_OK;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    if (n > g.regions_cap) {
        cudaFree(g.regions_dev);
        cudaFreeHost(g.regions_host);
        g.regions_dev = nullptr;
        g.regions_host = nullptr;
        OKV_CUDA_TRY(cudaMalloc((void **)&g.regions_dev, (size_t)n * sizeof(uint32_t *)));
        OKV_CUDA_TRY(cudaMallocHost((void **)&g.regions_host, (size_t)n * sizeof(uint32_t *)));
        g.regions_cap = n;
    }
    memcpy(g.regions_host, want.data(), (size_t)n * sizeof(uint32_t *));
    OKV_CUDA_TRY(cudaMemcpyAsync(g.regions_dev, g.regions_host, (size_t)n * sizeof(uint32_t *),
                                 cudaMemcpyHostToDevice, g.stream));
    g.regions_last = want;
    return ORCHKV_OK;
}

size_t region_alloc(size_t words)
{
    for (auto it = g.free_regions.begin(); it != g.free_regions.end(); ++it) {
        if (it->second >= words) {
            const size_t off = it->first, len = it->second;
            g.free_regions.erase(it);
            if (len > words) g.free_regions[off + words] = len - words;
            return off;
        }
    }
    return (size_t)-1;
}

void region_free(size_t off, size_t words)
{
    auto it = g.free_regions.emplace(off, words).first;
    auto nx = std::next(it);
    if (nx != g.free_regions.end() && it->first + it->second == nx->first) {
        it->second += nx->second;
        g.free_regions.erase(nx);
    }
    if (it != g.free_regions.begin()) {
        auto pv = std::prev(it);
        if (pv->first + pv->second == it->first) {
            pv->second += it->second;
            g.free_regions.erase(it);
        }
    }
}

void release_all()
{
    if (g.attached) {
        // the manager outlives the data plane: give it back its own stream
        // and stop data-plane kernels from writing its slots
        tm_set_stream(g.attached, nullptr);
        g.attached = nullptr;
        g.p.attached = 0;
    }
    if (g.copy) cudaStreamSynchronize(g.copy);
    if (g.copy_in) cudaStreamSynchronize(g.copy_in);
    if (g.unpack) cudaStreamSynchronize(g.unpack);
    if (g.stream) cudaStreamSynchronize(g.stream);
    fold_check_words();
    cudaFree(g.p.gpu_base);
    if (g.p.dram_base) cudaFreeHost(g.p.dram_base);
    cudaFree(g.dev_meta);
    cudaFree(g.bt);
    cudaFree(g.scratch);
    cudaFree(g.stage);
    cudaFree(g.regions_dev);
    cudaFreeHost(g.regions_host);
    cudaFreeHost(g.res);
    cudaFreeHost(g.h_ctr);
    cudaFreeHost(g.h_meta);
    cudaFree(g.ring);
    cudaFree(g.pring);
    cudaFree(g.scratch2);
    cudaFree(g.sort_mem);
    cudaFreeHost(g.h_runs);
    cudaFreeHost(g.h_runs2);
    if (g.h_cold) cudaFreeHost(g.h_cold);
    g.h_cold = nullptr;
    for (auto &e : g.ev_cold) if (e) { cudaEventDestroy(e); e = nullptr; }
    g.sort_mem = nullptr;
    g.h_runs = g.h_runs2 = nullptr;
    g.scratch2 = nullptr;
    g.scratch2_words = 0;
    for (auto &e : g.ev_copied) if (e) cudaEventDestroy(e);
    g.ev_copied.clear();
    for (auto &e : g.ev_pk) if (e) { cudaEventDestroy(e); e = nullptr; }
    for (auto &e : g.ev_up) if (e) { cudaEventDestroy(e); e = nullptr; }
    for (auto &e : g.ev_mig) if (e) { cudaEventDestroy(e); e = nullptr; }
    for (auto &e : g.ev_h2d) if (e) { cudaEventDestroy(e); e = nullptr; }
    for (auto &e : g.ev_unpacked) if (e) { cudaEventDestroy(e); e = nullptr; }
    if (g.ev_in_done) cudaEventDestroy(g.ev_in_done);
    if (g.ev_packed) cudaEventDestroy(g.ev_packed);
    g.ev_in_done = g.ev_packed = nullptr;
    if (g.copy) cudaStreamDestroy(g.copy);
    if (g.copy_in) cudaStreamDestroy(g.copy_in);
    if (g.unpack) cudaStreamDestroy(g.unpack);
    g.copy = g.copy_in = g.unpack = nullptr;
    g.ring = g.pring = nullptr;
    g.h_meta = nullptr;
    if (g.own) cudaStreamDestroy(g.own);
    g.p = PoolDev();
    g.dev_meta = nullptr;
    g.bt = nullptr;
    g.scratch = nullptr;
    g.stage = nullptr;
    g.stage_cap = 0;
    g.regions_dev = nullptr;
    g.regions_host = nullptr;
    g.regions_cap = 0;
    g.regions_last.clear();
    g.res = nullptr;
    g.h_ctr = nullptr;
    g.own = g.stream = nullptr;
    g.free_regions.clear();
    g.attached = nullptr;
    g.active_requests = 0;
}

int compat(kv_request_ctx_t *ctx, int op, uint32_t l, uint32_t h, uint32_t bi, uint32_t arg,
           uint32_t arg2 = 0)
{
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!ctx) return ORCHKV_ERR_NOT_FOUND;
    int rc = launch_compat_op(g.p, req_dev(ctx), op, l, h, bi, arg, arg2, g.res, g.stream);
    if (rc) return rc;
    int krc = 0;
    rc = sync_result(&krc);
    return rc ? rc : krc;
}

}  // namespace

// Access for the no-device-copy paths of other translation units.
cudaStream_t orchkv_stream_internal() { return g.stream; }

extern "C" {

int orchkv_init_ext(const orchkv_config_t *cfg, const orchkv_config_ext_t *ext)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (g.inited) return ORCHKV_ERR_ALREADY;
    if (!cfg) return ORCHKV_ERR_INVALID;
    const size_t e = dtype_size(cfg->dtype);
    const size_t slab = kv_block_data_bytes(cfg->tokens_per_block, cfg->d_head, cfg->dtype);
    if (e == 0 || slab == 0 || cfg->gpu_pool_bytes < slab || cfg->dram_pool_bytes < slab ||
        cfg->max_blocks_per_head == 0)
        return ORCHKV_ERR_INVALID;
    g.cfg = *cfg;
    g.device = cfg->gpu_device_id;
    snprintf(g.base_dir, sizeof(g.base_dir), "%s",
             cfg->orchfs_base_dir && cfg->orchfs_base_dir[0] ? cfg->orchfs_base_dir : "/dev/shm/orchkv");
    g.cfg.orchfs_base_dir = g.base_dir;
    mkdir_p(g.base_dir);
    g.storage_writes = g.storage_reads = 0;
    g.storage_bytes_written = g.storage_bytes_read = 0;
    // any early return below releases what was allocated so far
    struct InitGuard {
        bool ok = false;
        ~InitGuard() { if (!ok) release_all(); }
    } guard;
    OKV_CUDA_TRY(cudaSetDevice(g.device));
    // the library's own stream is a blocking one: unless the caller sets a
    // stream, its work is ordered with the legacy default stream (buffers a
    // caller fills or reads there need no extra synchronisation)
    OKV_CUDA_TRY(cudaStreamCreate(&g.own));
    g.stream = g.own;

    PoolDev &p = g.p;
    p = PoolDev();
    p.slab = slab;
    p.half = slab / 2;
    p.row = (uint32_t)(cfg->d_head * e);
    p.tpb = cfg->tokens_per_block;
    const uint64_t g_total = cfg->gpu_pool_bytes / slab, d_total = cfg->dram_pool_bytes / slab;
    if (g_total > kLocSlabMask || d_total > kLocSlabMask) return ORCHKV_ERR_INVALID;
    p.g_total = (uint32_t)g_total;
    p.d_total = (uint32_t)d_total;
    uint64_t mb = ext && ext->max_blocks ? ext->max_blocks : pow2_at_least(g_total + d_total);
    if (mb > 0x7FFFFFFFull) mb = 0x7FFFFFFFull;
    p.max_blocks = (uint32_t)mb;

    if (cudaMalloc((void **)&p.gpu_base, (size_t)p.g_total * slab) != cudaSuccess) {
        fprintf(stderr, "[orchkv] GPU pool allocation of %zu MB failed\n",
                ((size_t)p.g_total * slab) >> 20);
        release_all();
        return ORCHKV_ERR_CUDA;
    }
    // The DRAM tier must be pinned and mapped: migration kernels address it.
    if (cudaHostAlloc((void **)&p.dram_base, (size_t)p.d_total * slab,
                      cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
        fprintf(stderr, "[orchkv] pinned DRAM pool allocation of %zu MB failed\n",
                ((size_t)p.d_total * slab) >> 20);
        p.dram_base = nullptr;
        release_all();
        return ORCHKV_ERR_CUDA;
    }
    char *dram_dev = nullptr;
    if (cudaHostGetDevicePointer((void **)&dram_dev, p.dram_base, 0) != cudaSuccess ||
        dram_dev != p.dram_base) {
        fprintf(stderr, "[orchkv] DRAM pool is not addressable at its host address\n");
        release_all();
        return ORCHKV_ERR_CUDA;
    }

    const size_t meta = ((size_t)p.g_total + p.d_total + 2 * (size_t)p.max_blocks) * 4 +
                        (size_t)p.max_blocks * 6 + sizeof(PoolCounters) + 16 + 9 * 256;
    if (cudaMalloc((void **)&g.dev_meta, meta) != cudaSuccess) { release_all(); return ORCHKV_ERR_CUDA; }
    char *q = g.dev_meta;
    auto take = [&](size_t sz) { char *r = q; q += (sz + 255) & ~size_t(255); return r; };
    p.g_stack = (uint32_t *)take((size_t)p.g_total * 4);
    p.d_stack = (uint32_t *)take((size_t)p.d_total * 4);
    p.id_stack = (uint32_t *)take((size_t)p.max_blocks * 4);
    p.loc = (uint32_t *)take((size_t)p.max_blocks * 4);
    p.first = (uint32_t *)take((size_t)p.max_blocks * 4);
    p.state = (uint8_t *)take(p.max_blocks);
    p.flags = (uint8_t *)take(p.max_blocks);
    p.ctr = (PoolCounters *)take(sizeof(PoolCounters));
    p.chk = (uint32_t *)take(16);
    OKV_CUDA_TRY(cudaMemset(p.chk, 0, 16));

    // stacks hold N-1 ... 0 so the first pops return 0, 1, 2, ...
    // (src/tiered_store/gpu_tier.cu:41-42)
    {
        uint64_t mx = p.g_total > p.d_total ? p.g_total : p.d_total;
        if (p.max_blocks > mx) mx = p.max_blocks;
        std::vector<uint32_t> fill(mx);
        auto up = [&](uint32_t *dst, uint32_t n) -> int {
            for (uint32_t i = 0; i < n; i++) fill[i] = n - 1 - i;
            OKV_CUDA_TRY(cudaMemcpy(dst, fill.data(), (size_t)n * 4, cudaMemcpyHostToDevice));
            return ORCHKV_OK;
        };
        int rc = up(p.g_stack, p.g_total);
        if (!rc) rc = up(p.d_stack, p.d_total);
        if (!rc) rc = up(p.id_stack, p.max_blocks);
        if (rc) { release_all(); return rc; }
    }
    OKV_CUDA_TRY(cudaMemset(p.loc, 0xFF, (size_t)p.max_blocks * 4));  // tier 7: no block
    OKV_CUDA_TRY(cudaMemset(p.first, 0xFF, (size_t)p.max_blocks * 4));
    OKV_CUDA_TRY(cudaMemset(p.state, KV_STATE_EVICTED, p.max_blocks));
    OKV_CUDA_TRY(cudaMemset(p.flags, 0, p.max_blocks));
    PoolCounters c0;
    memset(&c0, 0, sizeof(c0));
    c0.g_top = p.g_total;
    c0.d_top = p.d_total;
    c0.id_top = p.max_blocks;
    OKV_CUDA_TRY(cudaMemcpy(p.ctr, &c0, sizeof(c0), cudaMemcpyHostToDevice));

    g.bt_words = ext && ext->table_entries ? ext->table_entries : (size_t)p.max_blocks * 2 + 65536;
    if (cudaMalloc((void **)&g.bt, g.bt_words * 4) != cudaSuccess) { release_all(); return ORCHKV_ERR_CUDA; }
    g.free_regions.clear();
    g.free_regions[0] = g.bt_words;
    g.scratch_words = (size_t)p.max_blocks * 3 + p.max_blocks / 1024 + 4096 +
                      (size_t)2 * (ext && ext->max_requests ? ext->max_requests : 4096) * 256;
    if (cudaMalloc((void **)&g.scratch, g.scratch_words * 4) != cudaSuccess) {
        release_all();
        return ORCHKV_ERR_CUDA;
    }
    OKV_CUDA_TRY(cudaMallocHost((void **)&g.res, sizeof(CompatResult)));
    OKV_CUDA_TRY(cudaMallocHost((void **)&g.h_ctr, sizeof(PoolCounters)));
    OKV_CUDA_TRY(cudaMallocHost((void **)&g.h_meta, 16 * 4));
    memset(g.res, 0, sizeof(CompatResult));
    OKV_CUDA_TRY(cudaStreamCreateWithFlags(&g.copy, cudaStreamNonBlocking));
    OKV_CUDA_TRY(cudaStreamCreateWithFlags(&g.copy_in, cudaStreamNonBlocking));
    OKV_CUDA_TRY(cudaStreamCreateWithFlags(&g.unpack, cudaStreamNonBlocking));
    g.ring_slabs = (uint32_t)(kChunkBytes / slab);
    if (g.ring_slabs == 0) g.ring_slabs = 1;
    {
        // evict staging: kRing slots by default; ext->staging_mb enlarges it so
        // a whole batch can be packed at once (what lets a swap overlap)
        const size_t slot_bytes = (size_t)g.ring_slabs * slab;
        size_t slots = ext && ext->staging_mb ? ((size_t)ext->staging_mb << 20) / slot_bytes : 0;
        if (slots < (size_t)kRing) slots = kRing;
        if (slots > (size_t)kMaxChunks) slots = kMaxChunks;
        if (cudaMalloc((void **)&g.ring, slots * slot_bytes) != cudaSuccess) {
            fprintf(stderr, "[orchkv] staging ring of %zu MB could not be allocated\n",
                    (slots * slot_bytes) >> 20);
            g.ring = nullptr;
            release_all();
            return ORCHKV_ERR_CUDA;
        }
        g.ev_copied.assign(slots, nullptr);
        OKV_CUDA_TRY(cudaMalloc((void **)&g.pring, (size_t)kRing * slot_bytes));
    }
    for (auto &e : g.ev_copied) OKV_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (auto &e : g.ev_pk) OKV_CUDA_TRY(cudaEventCreate(&e));
    for (auto &e : g.ev_up) OKV_CUDA_TRY(cudaEventCreate(&e));
    for (auto &e : g.ev_mig) OKV_CUDA_TRY(cudaEventCreate(&e));
    for (auto &e : g.ev_h2d) OKV_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    for (auto &e : g.ev_unpacked) OKV_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    OKV_CUDA_TRY(cudaEventCreateWithFlags(&g.ev_in_done, cudaEventDisableTiming));
    OKV_CUDA_TRY(cudaEventCreateWithFlags(&g.ev_packed, cudaEventDisableTiming));
    g.scratch2_words = (size_t)p.max_blocks * 3 + p.max_blocks / 1024 + 4096;
    OKV_CUDA_TRY(cudaMalloc((void **)&g.scratch2, g.scratch2_words * 4));
    {
        // two sort scratches over the DRAM pool: the evict's assignment and
        // the promote's source order (with its slab -> position map)
        const size_t dt = p.d_total, tiles = (dt + 1023) / 1024;
        const size_t one = dt * 2 + (tiles + dt + 2 * (size_t)kMaxRuns) * 4 + 8 * 256;
        const size_t bytes = 2 * one + dt * 4 + 256;
        OKV_CUDA_TRY(cudaMalloc((void **)&g.sort_mem, bytes));
        char *q2 = g.sort_mem;
        auto take2 = [&](size_t sz) { char *r = q2; q2 += (sz + 255) & ~size_t(255); return r; };
        for (SortScratch *x : {&g.ss, &g.ss2}) {
            x->flags = (uint8_t *)take2(dt);
            x->run_flag = (uint8_t *)take2(dt);
            x->tile_cnt = (uint32_t *)take2(tiles * 4);
            x->sorted = (uint32_t *)take2(dt * 4);
            x->run_o = (uint32_t *)take2((size_t)kMaxRuns * 4);
            x->run_d = (uint32_t *)take2((size_t)kMaxRuns * 4);
            x->max_runs = kMaxRuns;
            x->pos_of = nullptr;
        }
        g.ss2.pos_of = (uint32_t *)take2(dt * 4);
        OKV_CUDA_TRY(cudaMallocHost((void **)&g.h_runs, (size_t)kMaxRuns * 8));
        OKV_CUDA_TRY(cudaMallocHost((void **)&g.h_runs2, (size_t)kMaxRuns * 8));
    }
    g.active_requests = 0;
    g.inited = true;
    guard.ok = true;
    return ORCHKV_OK;
}

int orchkv_init(const orchkv_config_t *config) { return orchkv_init_ext(config, nullptr); }

int orchkv_shutdown(void)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    release_all();
    g.inited = false;
    return ORCHKV_OK;
}

bool orchkv_is_initialized(void) { return g.inited; }

kv_request_ctx_t *orchkv_request_create(uint64_t request_id, uint32_t n_layers,
                                        uint32_t n_kv_heads)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited || n_layers == 0 || n_kv_heads == 0) return nullptr;
    const uint32_t mbph = g.cfg.max_blocks_per_head;
    const size_t words = req_region_words(n_layers, n_kv_heads, mbph);
    const size_t off = region_alloc(words);
    if (off == (size_t)-1) return nullptr;
    kv_request_ctx_t *c = new (std::nothrow) kv_request_ctx_t();
    if (!c) { region_free(off, words); return nullptr; }
    c->request_id = request_id;
    c->L = n_layers;
    c->H = n_kv_heads;
    c->mbph = mbph;
    c->region_off = off;
    c->region_words = words;
    uint32_t *r = g.bt + off;
    if (cudaMemsetAsync(r, 0, (1 + n_layers) * 4, g.stream) != cudaSuccess ||
        cudaMemsetAsync(r + 1 + n_layers, 0xFF, (words - 1 - n_layers) * 4, g.stream) != cudaSuccess) {
        region_free(off, words);
        delete c;
        return nullptr;
    }
    // one storage file per request, as orchfs_file_open does
    // (src/tiered_store/orchfs_tier.c:201-230); a request without one still
    // works, its storage calls return ORCHKV_ERR_INIT
    snprintf(c->path, sizeof(c->path), "%s/req_%lu", g.base_dir, (unsigned long)request_id);
    c->fd = open(c->path, O_CREAT | O_RDWR, 0644);
    g.active_requests++;
    return c;
}

int orchkv_request_destroy(kv_request_ctx_t *ctx)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!ctx) return ORCHKV_ERR_INVALID;
    if (!g.inited) { delete ctx; return ORCHKV_ERR_INIT; }
    if ((size_t)3 * ((ctx->region_words + 1023) / 1024) > g.scratch_words) return ORCHKV_ERR_INVALID;
    int rc = launch_request_free(g.p, req_dev(ctx), g.scratch, g.stream);
    if (rc) return rc;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    if (ctx->fd >= 0) {                   // orchfs_file_close: close + unlink
        close(ctx->fd);
        unlink(ctx->path);
    }
    region_free(ctx->region_off, ctx->region_words);
    g.regions_last.clear();
    if (g.active_requests) g.active_requests--;
    delete ctx;
    return ORCHKV_OK;
}

int orchkv_prefill(kv_request_ctx_t *ctx, uint32_t layer, const void *k, const void *v,
                   uint32_t seq_len)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!ctx || layer >= ctx->L) return ORCHKV_ERR_INVALID;
    const size_t bytes = (size_t)ctx->H * seq_len * g.p.row;
    const char *kd, *vd;
    int rc = resolve_kv(k, v, bytes, &kd, &vd);
    if (rc) return rc;
    rc = launch_prefill(g.p, req_dev(ctx), layer, kd, vd, seq_len, g.scratch, g.res, g.stream);
    if (rc) return rc;
    int krc = 0;
    rc = sync_result(&krc);
    return rc ? rc : krc;
}

int orchkv_append_token(kv_request_ctx_t *ctx, uint32_t layer, const void *k, const void *v)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!ctx || layer >= ctx->L) return ORCHKV_ERR_INVALID;
    const size_t bytes = (size_t)ctx->H * g.p.row;
    const char *kd, *vd;
    int rc = resolve_kv(k, v, bytes, &kd, &vd);
    if (rc) return rc;
    rc = launch_append_one(g.p, req_dev(ctx), layer, kd, vd, g.res, g.stream);
    if (rc) return rc;
    int krc = 0;
    rc = sync_result(&krc);
    return rc ? rc : krc;
}

int orchkv_get_kv_block(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi,
                        void **k_out, void **v_out)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    // storage -> DRAM first, then DRAM -> GPU (src/api/orchkv_api.cu:321-349)
    int rc = compat(ctx, OP_INFO, l, h, bi, 0);
    if (rc) return rc;
    const uint32_t tier = loc_tier(g.res->loc);
    if (tier == TIER_NVM || tier == TIER_SSD) {
        rc = orchkv_promote_from_storage(ctx, l, h, bi);
        if (rc) return rc;
    }
    rc = compat(ctx, OP_GET, l, h, bi, 0);
    if (rc) return rc;
    if (k_out) *k_out = (void *)g.res->k_ptr;
    if (v_out) *v_out = (void *)g.res->v_ptr;
    return ORCHKV_OK;
}

int orchkv_evict_to_dram(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    return compat(ctx, OP_EVICT, l, h, bi, 0);
}

int orchkv_promote_to_gpu(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    return compat(ctx, OP_PROMOTE, l, h, bi, 0);
}

// ---- storage tier: one file per request, POSIX pwrite/pread at the
// reference's offsets (src/tiered_store/orchfs_tier.h:89-97,
// orchfs_tier.c:246-317).  The DRAM slab is pinned host memory, so the file
// IO reads and writes it directly.

static off_t storage_offset(const kv_request_ctx_t *c, uint32_t l, uint32_t h, uint32_t bi)
{
    const uint64_t head_linear = (uint64_t)l * c->H + h;
    return (off_t)((head_linear * c->mbph + bi) * g.p.slab);
}

static bool full_io(bool write, int fd, char *buf, size_t n, off_t off)
{
    while (n > 0) {
        const ssize_t r = write ? pwrite(fd, buf, n, off) : pread(fd, buf, n, off);
        if (r < 0) {
            if (errno == EINTR) continue;
            return false;
        }
        if (r == 0) return false;          // short read: the slab was never written
        buf += r;
        off += r;
        n -= (size_t)r;
    }
    return true;
}

int orchkv_evict_to_storage(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi)
{
    // src/api/orchkv_api.cu:432-466
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    int rc = compat(ctx, OP_INFO, l, h, bi, 0);
    if (rc) return rc;
    const uint32_t w = g.res->loc;
    if (loc_tier(w) != TIER_HOST_DRAM) return ORCHKV_ERR_STATE;
    if (g.res->flags & KV_FLAG_PIN) return ORCHKV_ERR_LOCKED;
    if (ctx->fd < 0) return ORCHKV_ERR_INIT;
    const uint32_t d = loc_slab(w);
    if (!full_io(true, ctx->fd, g.p.dram_base + (size_t)d * g.p.slab, g.p.slab,
                 storage_offset(ctx, l, h, bi)))
        return ORCHKV_ERR_IO;
    g.storage_writes++;
    g.storage_bytes_written += g.p.slab;
    // tier := NVM (the reference records file blocks as TIER_NVM), state COLD,
    // DRAM slab back to its pool
    return compat(ctx, OP_SET_LOC, l, h, bi, make_loc(TIER_NVM, 0),
                  (uint32_t)KV_STATE_COLD | ((d + 1) << 8));
}

int orchkv_promote_from_storage(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi)
{
    // src/api/orchkv_api.cu:470-504
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    int rc = compat(ctx, OP_INFO, l, h, bi, 0);
    if (rc) return rc;
    const uint32_t w = g.res->loc;
    if (loc_tier(w) != TIER_NVM && loc_tier(w) != TIER_SSD) return ORCHKV_ERR_STATE;
    if (ctx->fd < 0) return ORCHKV_ERR_INIT;
    rc = compat(ctx, OP_DRAM_POP, l, h, bi, 0);
    if (rc) return rc;
    const uint32_t d = g.res->aux;
    if (!full_io(false, ctx->fd, g.p.dram_base + (size_t)d * g.p.slab, g.p.slab,
                 storage_offset(ctx, l, h, bi))) {
        compat(ctx, OP_SET_LOC, l, h, bi, w, (uint32_t)KV_STATE_COLD | ((d + 1) << 8));
        return ORCHKV_ERR_IO;
    }
    g.storage_reads++;
    g.storage_bytes_read += g.p.slab;
    return compat(ctx, OP_SET_LOC, l, h, bi, make_loc(TIER_HOST_DRAM, d),
                  (uint32_t)KV_STATE_WARM);
}

int orchkv_evict_cold(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi)
{
    int rc = orchkv_evict_to_dram(ctx, l, h, bi);
    if (rc != ORCHKV_OK) return rc;
    return orchkv_evict_to_storage(ctx, l, h, bi);
}

void orchkv_storage_flush(void) {}

int orchkv_get_stats(orchkv_stats_t *s)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!s) return ORCHKV_ERR_INVALID;
    OKV_CUDA_TRY(cudaMemcpyAsync(g.h_ctr, g.p.ctr, sizeof(PoolCounters), cudaMemcpyDeviceToHost, g.stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    const PoolCounters &c = *g.h_ctr;
    memset(s, 0, sizeof(*s));
    s->gpu_pool_total = (size_t)g.p.g_total * g.p.slab;
    s->gpu_slabs_total = g.p.g_total;
    s->gpu_slabs_used = g.p.g_total - c.g_top;
    s->gpu_pool_used = (size_t)s->gpu_slabs_used * g.p.slab;
    s->dram_pool_total = (size_t)g.p.d_total * g.p.slab;
    s->dram_slabs_total = g.p.d_total;
    s->dram_slabs_used = g.p.d_total - c.d_top;
    s->dram_pool_used = (size_t)s->dram_slabs_used * g.p.slab;
    s->total_blocks = c.live_blocks;
    s->transfers_d2h = c.transfers_d2h;
    s->transfers_h2d = c.transfers_h2d;
    s->bytes_d2h = c.bytes_d2h;
    s->bytes_h2d = c.bytes_h2d;
    return ORCHKV_OK;
}

gpu_tier_t *orchkv_gpu_tier(void)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return nullptr;
    uint32_t top = 0;
    g.gsnap_stack.resize(g.p.g_total);
    if (orchkv_read_pool(0, g.gsnap_stack.data(), &top) != ORCHKV_OK) return nullptr;
    gpu_tier_t &t = g.gsnap;
    t.device_id = g.device;
    t.pool_base = g.p.gpu_base;
    t.pool_size = (size_t)g.p.g_total * g.p.slab;
    t.slab_size = g.p.slab;
    t.total_slabs = g.p.g_total;
    t.used_slabs = g.p.g_total - top;
    t.free_stack = g.gsnap_stack.data();
    t.free_top = top;
    return &t;
}

dram_tier_t *orchkv_dram_tier(void)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return nullptr;
    uint32_t top = 0;
    g.dsnap_stack.resize(g.p.d_total);
    if (orchkv_read_pool(1, g.dsnap_stack.data(), &top) != ORCHKV_OK) return nullptr;
    dram_tier_t &t = g.dsnap;
    t.pool_base = g.p.dram_base;
    t.pool_size = (size_t)g.p.d_total * g.p.slab;
    t.slab_size = g.p.slab;
    t.total_slabs = g.p.d_total;
    t.used_slabs = g.p.d_total - top;
    t.free_stack = g.dsnap_stack.data();
    t.free_top = top;
    t.is_pinned = true;
    return &t;
}

orchfs_tier_t *orchkv_orchfs_tier(void)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return nullptr;
    orchfs_tier_t &t = g.fsnap;
    t.initialized = true;
    snprintf(t.base_dir, sizeof(t.base_dir), "%s", g.base_dir);
    t.slab_size = g.p.slab;
    t.total_writes = g.storage_writes;
    t.total_reads = g.storage_reads;
    t.bytes_written = g.storage_bytes_written;
    t.bytes_read = g.storage_bytes_read;
    return &t;
}

// ---- B200 ------------------------------------------------------------------

int orchkv_set_stream(void *stream)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    g.stream = stream ? (cudaStream_t)stream : g.own;
    if (g.attached) tm_set_stream(g.attached, g.stream);
    return ORCHKV_OK;
}

int orchkv_sync(void)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    return check_words();
}

int orchkv_checked_build(void) { return kCheckedBuild ? 1 : 0; }

int orchkv_check_status(uint32_t *words, int reset)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!words) return ORCHKV_ERR_INVALID;
    if (g.inited) {
        OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
        const int rc = fold_check_words();
        if (rc) return rc;
    }
    memcpy(words, g_check_tally, sizeof(g_check_tally));
    if (reset) memset(g_check_tally, 0, sizeof(g_check_tally));
    return ORCHKV_OK;
}

int orchkv_check_inject(uint32_t line)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    return launch_check_inject(g.p, line, g.stream);
}

// Called by tm_sync: the data plane's check words (checked builds).
int okv_data_plane_check(void)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_OK;
    return check_words();
}

// Called by tm_destroy: a manager that goes away while attached is detached
// first, after the data-plane work queued against its slots has finished.
void okv_manager_destroyed(tiered_manager_t *tm)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited || g.attached != tm) return;
    tm_set_stream(tm, nullptr);
    g.attached = nullptr;
    g.p.attached = 0;
}

int orchkv_attach_scheduler(tiered_manager_t *tm)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!tm) {
        g.p.attached = 0;
        g.attached = nullptr;
        return ORCHKV_OK;
    }
    TmImpl *t = tm_impl(tm);
    if (!t) return ORCHKV_ERR_INVALID;
    if (t->cap < g.p.max_blocks) return ORCHKV_ERR_INVALID;
    int rc = tm_set_stream(tm, g.stream);
    if (rc) return rc;
    g.p.sd = t->d;
    g.p.attached = 1;
    g.attached = tm;
    return ORCHKV_OK;
}

int orchkv_append_token_batch(kv_request_ctx_t *const *ctxs, uint32_t n, const void *k,
                              const void *v)
{
    OKV_RANGE("orchkv_append_token_batch");
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    uint32_t L, H, mbph;
    int rc = upload_regions(ctxs, n, &L, &H, &mbph);
    if (rc) return rc;
    const size_t P = (size_t)n * L;
    if (2 * P + 16 > g.scratch_words) return ORCHKV_ERR_INVALID;
    const size_t bytes = P * H * g.p.row;
    const char *kd, *vd;
    rc = resolve_kv(k, v, bytes, &kd, &vd);
    if (rc) return rc;
    rc = launch_append_batch(g.p, g.regions_dev, n, L, H, mbph, kd, vd, g.scratch, g.stream);
    if (rc) return rc;
    // the all-or-nothing verdict is needed by the caller: read it back
    uint32_t err = 0;
    OKV_CUDA_TRY(cudaMemcpyAsync(&g.h_ctr->err, g.scratch + 2 * P, 4, cudaMemcpyDeviceToHost, g.stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    err = g.h_ctr->err;
    return (int)err;
}

}  // extern "C"

namespace {

// Pinned copies of a staged migration's metadata and run list.  false when
// nothing moved, or the runs do not fit kMaxRuns (the caller falls back).
bool read_runs(const MigPlan &mp, const SortScratch &ss, uint32_t *h_runs, uint32_t *done,
               uint32_t *n_runs, int *rc)
{
    *rc = ORCHKV_OK;
    if (cudaMemcpyAsync(g.h_meta, mp.meta, 8 * 4, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess ||
        cudaStreamSynchronize(g.stream) != cudaSuccess) {
        *rc = ORCHKV_ERR_CUDA;
        return false;
    }
    *done = g.h_meta[0];
    *n_runs = g.h_meta[6];
    if (*done == 0 || *n_runs == 0 || *n_runs > kMaxRuns) return false;
    if (cudaMemcpyAsync(h_runs, ss.run_o, (size_t)*n_runs * 4, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess ||
        cudaMemcpyAsync(h_runs + kMaxRuns, ss.run_d, (size_t)*n_runs * 4, cudaMemcpyDeviceToHost, g.stream) != cudaSuccess ||
        cudaStreamSynchronize(g.stream) != cudaSuccess) {
        *rc = ORCHKV_ERR_CUDA;
        return false;
    }
    return true;
}

// Runs shorter than this many slabs move zero-copy: per-copy overhead of the
// copy engine would exceed their transfer time.
uint32_t min_run_slabs(uint32_t done, uint32_t n_runs)
{
    uint32_t m = (uint32_t)((kCeMinRunBytes + g.p.slab - 1) / g.p.slab);
    if (m < 2) m = 2;
    return (n_runs == 1 && done >= m) ? 0 : m;   // 0: one long run, no per-entry lookups
}

// Drain a staged evict (after launch_sorted_assign and read_runs).  Runs of
// >= min_len slabs: pack into the ring at HBM speed, copy-engine D2H per run
// on g.copy.  Shorter runs: written zero-copy.  With pack_all (the whole
// batch fits the ring) every entry is packed before any drain and `packed`
// is recorded on g.stream after the last pack: from then on the victims' GPU
// slabs may be reused.  Returns with g.stream ordered after every drain.
int evict_drain(const MigPlan &mp, uint32_t done, uint32_t n_runs, bool pack_all,
                cudaEvent_t packed)
{
    const uint32_t *run_o = g.h_runs, *run_d = g.h_runs + kMaxRuns;
    const size_t slab = g.p.slab;
    const uint32_t min_len = min_run_slabs(done, n_runs);
    const uint32_t chunk = g.ring_slabs;
    const uint32_t nchunks = (done + chunk - 1) / chunk;
    const uint32_t slots = (uint32_t)g.ev_copied.size();
    if (nchunks > (uint32_t)kMaxChunks) return launch_migrate_zero_copy(g.p, 0, mp, g.stream);
    int rc;
    if (pack_all) {
        for (uint32_t c = 0; c < nchunks; c++) {
            const uint32_t pos0 = c * chunk, n = done - pos0 < chunk ? done - pos0 : chunk;
            OKV_CUDA_TRY(cudaEventRecord(g.ev_pk[2 * c], g.stream));
            rc = launch_pack(g.p, mp, g.ring + (size_t)c * chunk * slab, pos0, n, g.ss, 0, g.stream);
            if (rc) return rc;
            OKV_CUDA_TRY(cudaEventRecord(g.ev_pk[2 * c + 1], g.stream));
        }
        OKV_CUDA_TRY(cudaEventRecord(packed, g.stream));
    }
    uint32_t r = 0, ce_copies = 0, zc_slabs = 0;
    for (uint32_t c = 0; c < nchunks; c++) {
        const uint32_t slot = pack_all ? c : c % slots;
        const uint32_t pos0 = c * chunk;
        const uint32_t n = done - pos0 < chunk ? done - pos0 : chunk;
        char *buf = g.ring + (size_t)slot * chunk * slab;
        // list positions [pos0, pos0 + n) split into runs of consecutive slabs
        while (r + 1 < n_runs && run_o[r + 1] <= pos0) r++;
        uint32_t chunk_short = 0, q_end = r;
        for (uint32_t q = r; q < n_runs && run_o[q] < pos0 + n; q++) {
            const uint32_t run_end = q + 1 < n_runs ? run_o[q + 1] : done;
            const uint32_t a = run_o[q] > pos0 ? run_o[q] : pos0;
            const uint32_t b = run_end < pos0 + n ? run_end : pos0 + n;
            if (min_len && run_end - run_o[q] < min_len) chunk_short += b - a;
            q_end = q + 1;
        }
        if (!pack_all) {
            if (c >= slots) OKV_CUDA_TRY(cudaStreamWaitEvent(g.stream, g.ev_copied[slot], 0));
            OKV_CUDA_TRY(cudaEventRecord(g.ev_pk[2 * c], g.stream));
            if (chunk_short < n) {
                rc = launch_pack(g.p, mp, buf, pos0, n, g.ss, chunk_short ? min_len : 0, g.stream);
                if (rc) return rc;
            }
            OKV_CUDA_TRY(cudaEventRecord(g.ev_pk[2 * c + 1], g.stream));
        }
        OKV_CUDA_TRY(cudaStreamWaitEvent(g.copy, g.ev_pk[2 * c + 1], 0));
        for (uint32_t q = r; q < q_end; q++) {
            const uint32_t run_end = q + 1 < n_runs ? run_o[q + 1] : done;
            if (min_len && run_end - run_o[q] < min_len) continue;
            const uint32_t a = run_o[q] > pos0 ? run_o[q] : pos0;
            const uint32_t b = run_end < pos0 + n ? run_end : pos0 + n;
            const uint32_t d0 = run_d[q] + (a - run_o[q]);
            OKV_CUDA_TRY(cudaMemcpyAsync(g.p.dram_base + (size_t)d0 * slab,
                                         buf + (size_t)(a - pos0) * slab,
                                         (size_t)(b - a) * slab, cudaMemcpyDeviceToHost, g.copy));
            ce_copies++;
        }
        if (!pack_all) OKV_CUDA_TRY(cudaEventRecord(g.ev_copied[slot], g.copy));
        if (chunk_short) {
            rc = launch_drain_short(g.p, mp, pos0, n, g.ss, min_len, pack_all ? buf : nullptr,
                                    g.stream);
            if (rc) return rc;
            zc_slabs += chunk_short;
        }
    }
    // later work on the stream sees the bytes in the DRAM tier
    OKV_CUDA_TRY(cudaEventRecord(g.ev_mig[0], g.copy));
    OKV_CUDA_TRY(cudaStreamWaitEvent(g.stream, g.ev_mig[0], 0));
    g.last_evict_staged = 1;
    g.last_chunks = nchunks;
    g.last_pack_bytes = (unsigned long long)(pack_all ? done : done - zc_slabs) * slab * 2;
    g.last_runs = n_runs;
    g.last_ce_copies = ce_copies;
    g.last_zc_slabs = zc_slabs;
    return ORCHKV_OK;
}

// Zero-copy promote of a planned batch, timed by ev_mig[1..2].
int promote_zero_copy(const MigPlan &mp)
{
    OKV_CUDA_TRY(cudaEventRecord(g.ev_mig[1], g.stream));
    int rc = launch_migrate_zero_copy(g.p, 1, mp, g.stream);
    OKV_CUDA_TRY(cudaEventRecord(g.ev_mig[2], g.stream));
    g.last_promote_timed = 1;
    return rc;
}

// Drain a staged promote (after launch_sorted_sources on g.ss2 and
// read_runs into g.h_runs2).  Runs of >= min_len source slabs: copy-engine
// H2D into the promote ring on g.copy_in, scattered by unpack kernels on
// g.unpack; shorter runs: one zero-copy kernel.  `dram_ready` (may be null)
// gates every read of the DRAM tier, `gpu_ready` (may be null) every write
// into GPU slabs.  Returns with g.stream ordered after the whole promote.
int promote_drain(const MigPlan &mp, uint32_t done, uint32_t n_runs, cudaEvent_t dram_ready,
                  cudaEvent_t gpu_ready)
{
    const uint32_t *run_o = g.h_runs2, *run_d = g.h_runs2 + kMaxRuns;
    const size_t slab = g.p.slab;
    const uint32_t min_len = min_run_slabs(done, n_runs);
    const uint32_t chunk = g.ring_slabs;
    const uint32_t nchunks = (done + chunk - 1) / chunk;
    if (nchunks > (uint32_t)kMaxChunks) return promote_zero_copy(mp);
    if (dram_ready) {
        OKV_CUDA_TRY(cudaStreamWaitEvent(g.copy_in, dram_ready, 0));
        OKV_CUDA_TRY(cudaStreamWaitEvent(g.unpack, dram_ready, 0));
    }
    if (gpu_ready) OKV_CUDA_TRY(cudaStreamWaitEvent(g.unpack, gpu_ready, 0));
    OKV_CUDA_TRY(cudaEventRecord(g.ev_mig[1], g.copy_in));
    int rc;
    uint32_t r = 0, ce_copies = 0, zc_slabs = 0;
    for (uint32_t c = 0; c < nchunks; c++) {
        const uint32_t slot = c % kRing;
        const uint32_t j0 = c * chunk;
        const uint32_t n = done - j0 < chunk ? done - j0 : chunk;
        char *buf = g.pring + (size_t)slot * chunk * slab;
        while (r + 1 < n_runs && run_o[r + 1] <= j0) r++;
        uint32_t chunk_long = 0, q_end = r;
        for (uint32_t q = r; q < n_runs && run_o[q] < j0 + n; q++) {
            const uint32_t run_end = q + 1 < n_runs ? run_o[q + 1] : done;
            const uint32_t a = run_o[q] > j0 ? run_o[q] : j0;
            const uint32_t b = run_end < j0 + n ? run_end : j0 + n;
            if (min_len && run_end - run_o[q] < min_len) zc_slabs += b - a;
            else chunk_long += b - a;
            q_end = q + 1;
        }
        if (chunk_long == 0) continue;
        if (c >= (uint32_t)kRing) OKV_CUDA_TRY(cudaStreamWaitEvent(g.copy_in, g.ev_unpacked[slot], 0));
        for (uint32_t q = r; q < q_end; q++) {
            const uint32_t run_end = q + 1 < n_runs ? run_o[q + 1] : done;
            if (min_len && run_end - run_o[q] < min_len) continue;
            const uint32_t a = run_o[q] > j0 ? run_o[q] : j0;
            const uint32_t b = run_end < j0 + n ? run_end : j0 + n;
            const uint32_t s0 = run_d[q] + (a - run_o[q]);
            OKV_CUDA_TRY(cudaMemcpyAsync(buf + (size_t)(a - j0) * slab,
                                         g.p.dram_base + (size_t)s0 * slab,
                                         (size_t)(b - a) * slab, cudaMemcpyHostToDevice, g.copy_in));
            ce_copies++;
        }
        OKV_CUDA_TRY(cudaEventRecord(g.ev_h2d[c], g.copy_in));
        OKV_CUDA_TRY(cudaStreamWaitEvent(g.unpack, g.ev_h2d[c], 0));
        const uint32_t u = g.last_unpacks;                     // < kMaxChunks: timed
        if (u < (uint32_t)kMaxChunks) OKV_CUDA_TRY(cudaEventRecord(g.ev_up[2 * u], g.unpack));
        rc = launch_unpack(g.p, mp, g.ss2, buf, j0, n, min_len, g.unpack);
        if (rc) return rc;
        if (u < (uint32_t)kMaxChunks) {
            OKV_CUDA_TRY(cudaEventRecord(g.ev_up[2 * u + 1], g.unpack));
            g.last_unpack_bytes[u] = 2ull * chunk_long * slab;  // ring read + GPU slab write
            g.last_unpacks = u + 1;
        }
        OKV_CUDA_TRY(cudaEventRecord(g.ev_unpacked[slot], g.unpack));
    }
    if (zc_slabs) {
        rc = launch_promote_short(g.p, mp, g.ss2, min_len, g.unpack);
        if (rc) return rc;
    }
    OKV_CUDA_TRY(cudaEventRecord(g.ev_in_done, g.copy_in));
    OKV_CUDA_TRY(cudaStreamWaitEvent(g.unpack, g.ev_in_done, 0));
    OKV_CUDA_TRY(cudaEventRecord(g.ev_mig[2], g.unpack));
    OKV_CUDA_TRY(cudaStreamWaitEvent(g.stream, g.ev_mig[2], 0));
    g.last_promote_timed = 1;
    g.last_p_runs = n_runs;
    g.last_p_ce_copies = ce_copies;
    g.last_p_zc_slabs = zc_slabs;
    return ORCHKV_OK;
}

void reset_profile()
{
    g.last_evict_staged = 0;
    g.last_chunks = 0;
    g.last_pack_bytes = 0;
    g.last_runs = g.last_ce_copies = g.last_zc_slabs = 0;
    g.last_p_runs = g.last_p_ce_copies = g.last_p_zc_slabs = 0;
    g.last_swap_overlapped = 0;
    g.last_swap_conflicts = 0;
    g.last_unpacks = 0;
}

bool scratch_fits(uint32_t max_n)
{
    return (size_t)3 * max_n + max_n / 1024 + 32 <= g.scratch_words;
}

// Evict a planned batch: staged when large, else the fused zero-copy kernel.
int evict_planned(const MigPlan &mp, uint32_t max_n)
{
    if (max_n >= kStagedMin) {
        int rc = launch_sorted_assign(g.p, mp, g.ss, g.stream);
        if (rc) return rc;
        uint32_t done = 0, n_runs = 0;
        if (read_runs(mp, g.ss, g.h_runs, &done, &n_runs, &rc))
            return evict_drain(mp, done, n_runs, false, nullptr);
        if (rc || done == 0) return rc;
    }
    return launch_migrate_zero_copy(g.p, 0, mp, g.stream);
}

// Promote a planned batch: staged when large (copy engine for long source
// runs), else the fused zero-copy kernel.
int promote_planned(const MigPlan &mp, uint32_t max_n, cudaEvent_t ready)
{
    if (max_n >= kStagedMin) {
        int rc = launch_sorted_sources(g.p, mp, g.ss2, g.stream);
        if (rc) return rc;
        uint32_t done = 0, n_runs = 0;
        if (read_runs(mp, g.ss2, g.h_runs2, &done, &n_runs, &rc))
            return promote_drain(mp, done, n_runs, ready, ready);
        if (rc || done == 0) return rc;
    }
    return promote_zero_copy(mp);
}

}  // namespace

extern "C" {

int orchkv_evict_batch_to_dram(const uint32_t *ids, const uint32_t *count, uint32_t max_n,
                               uint32_t *result)
{
    OKV_RANGE("orchkv_evict_batch_to_dram");
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (max_n && !ids) return ORCHKV_ERR_INVALID;
    if (!scratch_fits(max_n)) return ORCHKV_ERR_INVALID;
    reset_profile();
    MigPlan mp = launch_migrate_plan(g.p, 0, ids, count, max_n, result, g.scratch, g.stream);
    if (mp.rc) return mp.rc;
    // Large batch: the DRAM slabs popped for it are sorted and handed out in
    // ascending order; victims are packed into a device staging ring at HBM
    // speed and the copy engine drains each slot into the DRAM tier, one copy
    // per run of consecutive slabs, while the next slot is packed.  Pool
    // stacks end exactly as after per-block evicts; only which victim gets
    // which of the popped slabs differs.
    return evict_planned(mp, max_n);
}

int orchkv_promote_batch_to_gpu(const uint32_t *ids, const uint32_t *count, uint32_t max_n,
                                uint32_t *result)
{
    OKV_RANGE("orchkv_promote_batch_to_gpu");
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (max_n && !ids) return ORCHKV_ERR_INVALID;
    if (!scratch_fits(max_n)) return ORCHKV_ERR_INVALID;
    reset_profile();
    MigPlan mp = launch_migrate_plan(g.p, 1, ids, count, max_n, result, g.scratch, g.stream);
    if (mp.rc) return mp.rc;
    // Sources are wherever the blocks sit in the DRAM tier: sorted, long runs
    // of consecutive slabs go through the copy engine (H2D + unpack), the
    // rest is read zero-copy by one kernel.
    return promote_planned(mp, max_n, nullptr);
}

int orchkv_swap_batch(const uint32_t *evict_ids, const uint32_t *evict_count, uint32_t max_e,
                      const uint32_t *promote_ids, const uint32_t *promote_count,
                      uint32_t max_p, uint32_t *result)
{
    OKV_RANGE("orchkv_swap_batch");
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if ((max_e && !evict_ids) || (max_p && !promote_ids)) return ORCHKV_ERR_INVALID;
    if (!scratch_fits(max_e) || (size_t)3 * max_p + max_p / 1024 + 32 > g.scratch2_words)
        return ORCHKV_ERR_INVALID;
    reset_profile();
    // Plans in call order: the evict's pops and pushes (and its sorted DRAM
    // assignment) first, then the promote's, so stacks and locations end as
    // after the evict list followed by the promote list, block by block.
    MigPlan me = launch_migrate_plan(g.p, 0, evict_ids, evict_count, max_e, result, g.scratch,
                                     g.stream);
    if (me.rc) return me.rc;
    const bool staged_e = max_e >= kStagedMin;
    int rc;
    if (staged_e) {
        rc = launch_sorted_assign(g.p, me, g.ss, g.stream);
        if (rc) return rc;
    }
    MigPlan mq = launch_migrate_plan(g.p, 1, promote_ids, promote_count, max_p,
                                     result ? result + 2 : nullptr, g.scratch2, g.stream);
    if (mq.rc) return mq.rc;
    const bool staged_p = max_p >= kStagedMin;
    if (staged_p) {
        rc = launch_sorted_sources(g.p, mq, g.ss2, g.stream);
        if (rc) return rc;
    }
    uint32_t de = 0, re = 0, dq = 0, rq = 0;
    bool runs_e = false, runs_p = false;
    if (staged_e) {
        runs_e = read_runs(me, g.ss, g.h_runs, &de, &re, &rc);
        if (rc) return rc;
    }
    if (staged_p) {
        runs_p = read_runs(mq, g.ss2, g.h_runs2, &dq, &rq, &rc);
        if (rc) return rc;
    }
    // Overlap needs (a) every victim packed before the promote writes GPU
    // slabs the evict freed (the batch fits the ring) and (b) no promoted
    // block read from a DRAM slab this evict is still filling.
    bool overlap = runs_e && runs_p && (de + g.ring_slabs - 1) / g.ring_slabs <= g.ev_copied.size();
    if (overlap) {
        rc = launch_conflicts(g.p, mq, g.ss, g.h_meta + 8, g.stream);
        if (rc) return rc;
        OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
        g.last_swap_conflicts = g.h_meta[8];
        overlap = g.h_meta[8] == 0;
    }
    if (overlap) {
        // evict D2H and promote H2D run at once on the two copy engines
        rc = evict_drain(me, de, re, true, g.ev_packed);
        if (rc) return rc;
        rc = promote_drain(mq, dq, rq, nullptr, g.ev_packed);
        if (rc) return rc;
        g.last_swap_overlapped = 1;
        return ORCHKV_OK;
    }
    // one after the other
    if (runs_e) rc = evict_drain(me, de, re, false, nullptr);
    else rc = launch_migrate_zero_copy(g.p, 0, me, g.stream);
    if (rc) return rc;
    OKV_CUDA_TRY(cudaEventRecord(g.ev_packed, g.stream));
    if (runs_p) return promote_drain(mq, dq, rq, g.ev_packed, g.ev_packed);
    return promote_zero_copy(mq);
}

/* Timing of the last batched evict / promote / swap (synchronises the
 * stream): pack_ms = summed device time of the evict's pack kernels (0 if
 * the zero-copy path ran), pack_bytes = bytes they read + wrote, chunks =
 * staging slots used, promote_ms = device time of the promote, from its
 * first copy or kernel to its last. */
int orchkv_last_migration_profile(float *pack_ms, unsigned long long *pack_bytes,
                                  uint32_t *chunks, float *promote_ms)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    float total = 0.f;
    if (g.last_evict_staged) {
        for (uint32_t c = 0; c < g.last_chunks; c++) {
            float ms = 0.f;
            OKV_CUDA_TRY(cudaEventElapsedTime(&ms, g.ev_pk[2 * c], g.ev_pk[2 * c + 1]));
            total += ms;
        }
    }
    if (pack_ms) *pack_ms = total;
    if (pack_bytes) *pack_bytes = g.last_evict_staged ? g.last_pack_bytes : 0;
    if (chunks) *chunks = g.last_evict_staged ? g.last_chunks : 0;
    if (promote_ms) {
        *promote_ms = 0.f;
        if (g.last_promote_timed)
            OKV_CUDA_TRY(cudaEventElapsedTime(promote_ms, g.ev_mig[1], g.ev_mig[2]));
    }
    return ORCHKV_OK;
}

int orchkv_last_unpack_chunks(float *ms, unsigned long long *bytes, uint32_t max_launches,
                              uint32_t *launches)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    const uint32_t n = g.last_unpacks;
    if (launches) *launches = n;
    for (uint32_t u = 0; u < n && u < max_launches; u++) {
        if (ms) OKV_CUDA_TRY(cudaEventElapsedTime(&ms[u], g.ev_up[2 * u], g.ev_up[2 * u + 1]));
        if (bytes) bytes[u] = g.last_unpack_bytes[u];
    }
    return ORCHKV_OK;
}

int orchkv_last_pack_chunks(float *ms, uint32_t max_chunks, uint32_t *chunks)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    const uint32_t n = g.last_evict_staged ? g.last_chunks : 0;
    if (chunks) *chunks = n;
    for (uint32_t c = 0; ms && c < n && c < max_chunks; c++)
        OKV_CUDA_TRY(cudaEventElapsedTime(&ms[c], g.ev_pk[2 * c], g.ev_pk[2 * c + 1]));
    return ORCHKV_OK;
}

int orchkv_last_evict_layout(uint32_t *runs, uint32_t *ce_copies, uint32_t *zero_copy_slabs)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (runs) *runs = g.last_evict_staged ? g.last_runs : 0;
    if (ce_copies) *ce_copies = g.last_evict_staged ? g.last_ce_copies : 0;
    if (zero_copy_slabs) *zero_copy_slabs = g.last_evict_staged ? g.last_zc_slabs : 0;
    return ORCHKV_OK;
}

int orchkv_last_promote_layout(uint32_t *runs, uint32_t *ce_copies, uint32_t *zero_copy_slabs,
                               int *overlapped)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (runs) *runs = g.last_p_runs;
    if (ce_copies) *ce_copies = g.last_p_ce_copies;
    if (zero_copy_slabs) *zero_copy_slabs = g.last_p_zc_slabs;
    if (overlapped) *overlapped = g.last_swap_overlapped;
    return ORCHKV_OK;
}

// ---- batched storage moves ----------------------------------------------------

namespace {

constexpr size_t kStorageRunBytes = 1u << 20;   // one pwritev / preadv moves up to 1 MiB

struct LhbEntry {
    uint32_t pos;        // list position
    uint32_t id, slab;   // block id, DRAM slab
    off_t off;           // file offset (reference layout)
};

// Look up a request's (layer, head, block) triples: host out[3n] =
// {id, loc word, flags} per entry.
int lookup_lhb(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n, std::vector<uint32_t> &out)
{
    if ((size_t)6 * n + 32 > g.scratch_words) return ORCHKV_ERR_INVALID;
    uint32_t *d_in = g.scratch, *d_out = g.scratch + (size_t)3 * n;
    OKV_CUDA_TRY(cudaMemcpyAsync(d_in, lhb, (size_t)12 * n, cudaMemcpyHostToDevice, g.stream));
    int rc = launch_lhb_lookup(g.p, req_dev(ctx), d_in, n, d_out, g.stream);
    if (rc) return rc;
    out.resize((size_t)3 * n);
    OKV_CUDA_TRY(cudaMemcpyAsync(out.data(), d_out, (size_t)12 * n, cudaMemcpyDeviceToHost, g.stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    return ORCHKV_OK;
}

// One pwritev / preadv run: k buffers at consecutive file offsets from off0,
// resumed after short transfers (the iovecs are consumed).
bool io_run(bool write, int fd, iovec *v, int cnt, off_t off0)
{
    size_t done = 0, left = 0;
    for (int j = 0; j < cnt; j++) left += v[j].iov_len;
    while (left > 0) {
        const ssize_t r = write ? pwritev(fd, v, cnt, off0 + (off_t)done)
                                : preadv(fd, v, cnt, off0 + (off_t)done);
        if (r < 0) {
            if (errno == EINTR) continue;
            return false;
        }
        if (r == 0) return false;      // short read: a slab that was never written
        done += (size_t)r;
        left -= (size_t)r;
        size_t adv = (size_t)r;
        while (cnt > 0 && adv >= v->iov_len) { adv -= v->iov_len; v++; cnt--; }
        if (cnt > 0 && adv) {
            v->iov_base = (char *)v->iov_base + adv;
            v->iov_len -= adv;
        }
    }
    return true;
}

struct IoRun {
    off_t off;           // file offset of the first buffer
    size_t first, n;     // iovecs [first, first + n)
};

// Runs of a batch, in offset order.  Reads are spread over the configured IO
// workers (the reference's orchfs_io_workers, its IO worker pool size,
// src/tiered_store/io_worker.c:52-133): each worker takes the next run until
// all are done or one fails; runs read disjoint file ranges into disjoint
// buffers, so their order does not matter.  Writes stay on the calling
// thread: writers into one file queue on the file's lock in the kernel, and
// on a B200 box's tmpfs a 0.8 GB scattered two-hop evict wrote at 2.0 GB/s
// with one thread against 1.8 with four and 1.3 with sixteen, while reading
// it back ran at 4.7, 14.7 and 35.4 GB/s.
bool io_runs(bool write, int fd, std::vector<iovec> &iov, const std::vector<IoRun> &runs)
{
    std::atomic<size_t> next{0};
    std::atomic<bool> ok{true};
    auto work = [&]() {
        for (size_t r = next++; r < runs.size() && ok.load(); r = next++)
            if (!io_run(write, fd, iov.data() + runs[r].first, (int)runs[r].n, runs[r].off))
                ok = false;
    };
    size_t workers = g.cfg.orchfs_io_workers > 0 ? (size_t)g.cfg.orchfs_io_workers : 1;
    if (write) workers = 1;
    if (workers > 64) workers = 64;
    if (workers > runs.size()) workers = runs.size();
    std::vector<std::thread> pool;
    for (size_t t = 1; t < workers; t++) pool.emplace_back(work);
    work();
    for (auto &t : pool) t.join();
    return ok.load();
}

// Runs of consecutive file offsets (up to kStorageRunBytes each) over
// entries sorted by offset; bufs[j] is entry j's buffer.
void plan_runs(const std::vector<off_t> &offs, const std::vector<char *> &bufs, size_t slab,
               std::vector<iovec> &iov, std::vector<IoRun> &runs)
{
    size_t per_call = kStorageRunBytes / slab;
    if (per_call < 1) per_call = 1;
    if (per_call > (size_t)IOV_MAX) per_call = IOV_MAX;
    iov.resize(offs.size());
    runs.clear();
    for (size_t i = 0; i < offs.size();) {
        size_t k = 0;
        while (i + k < offs.size() && k < per_call && offs[i + k] == offs[i] + (off_t)(k * slab)) {
            iov[i + k].iov_base = bufs[i + k];
            iov[i + k].iov_len = slab;
            k++;
        }
        runs.push_back(IoRun{offs[i], i, k});
        i += k;
    }
}

// Write (evict) or read (promote) entries between their DRAM slabs and the
// request's file: sorted by file offset, consecutive offsets go out in one
// pwritev / preadv of up to kStorageRunBytes, straight from / into the
// slabs, the runs spread over the IO workers.
bool storage_io(bool write, int fd, std::vector<LhbEntry> e)
{
    std::sort(e.begin(), e.end(), [](const LhbEntry &a, const LhbEntry &b) { return a.off < b.off; });
    const size_t slab = g.p.slab;
    std::vector<off_t> offs(e.size());
    std::vector<char *> bufs(e.size());
    for (size_t j = 0; j < e.size(); j++) {
        offs[j] = e[j].off;
        bufs[j] = g.p.dram_base + (size_t)e[j].slab * slab;
    }
    std::vector<iovec> iov;
    std::vector<IoRun> runs;
    plan_runs(offs, bufs, slab, iov, runs);
    return io_runs(write, fd, iov, runs);
}

// Upload the committed entries (list order) and apply them on the device.
int storage_commit(const std::vector<LhbEntry> &e, int dir)
{
    const size_t n = e.size();
    if (n == 0) return ORCHKV_OK;
    std::vector<uint32_t> h(2 * n);
    for (size_t j = 0; j < n; j++) {
        h[j] = e[j].id;
        h[n + j] = e[j].slab;
    }
    OKV_CUDA_TRY(cudaMemcpyAsync(g.scratch, h.data(), 8 * n, cudaMemcpyHostToDevice, g.stream));
    int rc = launch_storage_commit(g.p, g.scratch, g.scratch + n, (uint32_t)n, dir, g.stream);
    if (rc) return rc;
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    return ORCHKV_OK;
}

// Entries of `lhb` on `tier` (and not pinned, for evicts), first occurrence
// of each block only, in list order.
std::vector<LhbEntry> pick(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n,
                           const std::vector<uint32_t> &look, bool from_dram)
{
    std::vector<LhbEntry> v;
    std::unordered_set<uint32_t> seen;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t id = look[3 * i], w = look[3 * i + 1], f = look[3 * i + 2];
        if (id == kNoBlock || !seen.insert(id).second) continue;
        const uint32_t t = loc_tier(w);
        if (from_dram ? (t != TIER_HOST_DRAM || (f & KV_FLAG_PIN))
                      : (t != TIER_NVM && t != TIER_SSD))
            continue;
        v.push_back(LhbEntry{i, id, loc_slab(w),
                             storage_offset(ctx, lhb[3 * i], lhb[3 * i + 1], lhb[3 * i + 2])});
    }
    return v;
}

int evict_batch_to_storage_locked(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n,
                                  uint32_t *result)
{
    if (result) { result[0] = 0; result[1] = n; }
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!ctx || (n && !lhb)) return ORCHKV_ERR_INVALID;
    if (n == 0) return ORCHKV_OK;
    if (ctx->fd < 0) return ORCHKV_ERR_INIT;
    std::vector<uint32_t> look;
    int rc = lookup_lhb(ctx, lhb, n, look);
    if (rc) return rc;
    std::vector<LhbEntry> e = pick(ctx, lhb, n, look, true);
    if (!storage_io(true, ctx->fd, e)) return ORCHKV_ERR_IO;
    rc = storage_commit(e, 0);
    if (rc) return rc;
    g.storage_writes += e.size();
    g.storage_bytes_written += e.size() * g.p.slab;
    if (result) { result[0] = (uint32_t)e.size(); result[1] = n - (uint32_t)e.size(); }
    return ORCHKV_OK;
}

}  // namespace

int orchkv_evict_batch_to_storage(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n,
                                  uint32_t *result)
{
    OKV_RANGE("orchkv_evict_batch_to_storage");
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    return evict_batch_to_storage_locked(ctx, lhb, n, result);
}

int orchkv_promote_batch_from_storage(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n,
                                      uint32_t *result)
{
    OKV_RANGE("orchkv_promote_batch_from_storage");
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (result) { result[0] = 0; result[1] = n; }
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!ctx || (n && !lhb)) return ORCHKV_ERR_INVALID;
    if (n == 0) return ORCHKV_OK;
    if (ctx->fd < 0) return ORCHKV_ERR_INIT;
    std::vector<uint32_t> look;
    int rc = lookup_lhb(ctx, lhb, n, look);
    if (rc) return rc;
    std::vector<LhbEntry> e = pick(ctx, lhb, n, look, false);
    // each promote pops the DRAM stack's top slab, in list order; once it is
    // empty the rest are skipped (ORCHKV_ERR_TIER_FULL per block)
    OKV_CUDA_TRY(cudaMemcpyAsync(g.h_ctr, g.p.ctr, sizeof(PoolCounters), cudaMemcpyDeviceToHost,
                                 g.stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    const uint32_t top = g.h_ctr->d_top;
    if (e.size() > top) e.resize(top);
    if (!e.empty()) {
        std::vector<uint32_t> pops(e.size());
        OKV_CUDA_TRY(cudaMemcpyAsync(pops.data(), g.p.d_stack + (top - e.size()),
                                     4 * e.size(), cudaMemcpyDeviceToHost, g.stream));
        OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
        for (size_t j = 0; j < e.size(); j++) e[j].slab = pops[e.size() - 1 - j];
    }
    if (!storage_io(false, ctx->fd, e)) return ORCHKV_ERR_IO;
    rc = storage_commit(e, 1);
    if (rc) return rc;
    g.storage_reads += e.size();
    g.storage_bytes_read += e.size() * g.p.slab;
    if (result) { result[0] = (uint32_t)e.size(); result[1] = n - (uint32_t)e.size(); }
    return ORCHKV_OK;
}

int orchkv_evict_cold_batch(kv_request_ctx_t *ctx, const uint32_t *lhb, uint32_t n,
                            uint32_t *result)
{
    OKV_RANGE("orchkv_evict_cold_batch");
    // per block, orchkv_evict_cold = orchkv_evict_to_dram then
    // orchkv_evict_to_storage (src/api/orchkv_api.cu:508-516): a GPU block
    // passes through the DRAM stack's top slab and the slab goes back, so a
    // run of them leaves the DRAM stack as it was and pushes the GPU slabs in
    // list order.  Here the victims are gathered (zero-copy) into a pinned
    // staging buffer and written from there.
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (result) { result[0] = 0; result[1] = n; }
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!ctx || (n && !lhb)) return ORCHKV_ERR_INVALID;
    if (n == 0) return ORCHKV_OK;
    std::vector<uint32_t> look;
    int rc = lookup_lhb(ctx, lhb, n, look);
    if (rc) return rc;
    std::vector<LhbEntry> e;
    std::unordered_set<uint32_t> seen;
    for (uint32_t i = 0; i < n; i++) {
        const uint32_t id = look[3 * i], w = look[3 * i + 1], f = look[3 * i + 2];
        if (id == kNoBlock || !seen.insert(id).second) continue;
        if (loc_tier(w) != TIER_GPU_HBM || (f & KV_FLAG_PIN)) continue;
        e.push_back(LhbEntry{i, id, loc_slab(w),
                             storage_offset(ctx, lhb[3 * i], lhb[3 * i + 1], lhb[3 * i + 2])});
    }
    if (e.empty()) return ORCHKV_OK;
    if (ctx->fd < 0) return ORCHKV_ERR_INIT;
    OKV_CUDA_TRY(cudaMemcpyAsync(g.h_ctr, g.p.ctr, sizeof(PoolCounters), cudaMemcpyDeviceToHost,
                                 g.stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    if (g.h_ctr->d_top == 0) return ORCHKV_OK;      // no DRAM slab to pass through: TIER_FULL
    // stage in file-offset order, in chunks of the pinned staging buffer:
    // two halves, so chunk c + 1 is gathered on the GPU while the IO workers
    // write chunk c from the other half
    std::vector<LhbEntry> io = e;
    std::sort(io.begin(), io.end(), [](const LhbEntry &a, const LhbEntry &b) { return a.off < b.off; });
    const size_t slab = g.p.slab;
    const uint32_t chunk = g.ring_slabs;
    if (!g.h_cold) OKV_CUDA_TRY(cudaHostAlloc((void **)&g.h_cold, 2 * (size_t)chunk * slab,
                                              cudaHostAllocMapped | cudaHostAllocPortable));
    if (!g.ev_cold[0])
        for (auto &ev : g.ev_cold)
            OKV_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    char *h_cold_dev = nullptr;
    OKV_CUDA_TRY(cudaHostGetDevicePointer((void **)&h_cold_dev, g.h_cold, 0));
    if ((size_t)2 * chunk + 16 > g.scratch_words) return ORCHKV_ERR_INVALID;
    std::vector<uint32_t> src[2] = {std::vector<uint32_t>(chunk), std::vector<uint32_t>(chunk)};
    const size_t n_chunks = (io.size() + chunk - 1) / chunk;
    auto gather = [&](size_t c) -> int {        // chunk c -> staging half c % 2
        const size_t c0 = c * chunk, h = c % 2;
        const uint32_t k = (uint32_t)std::min<size_t>(chunk, io.size() - c0);
        for (uint32_t j = 0; j < k; j++) src[h][j] = io[c0 + j].slab;
        OKV_CUDA_TRY(cudaMemcpyAsync(g.scratch + h * chunk, src[h].data(), (size_t)4 * k,
                                     cudaMemcpyHostToDevice, g.stream));
        MigPlan gp{};
        gp.plan_src = g.scratch + h * chunk;
        gp.max_n = k;
        const int r = launch_pack(g.p, gp, h_cold_dev + h * (size_t)chunk * slab, 0, k, g.ss, 0,
                                  g.stream);
        if (r) return r;
        OKV_CUDA_TRY(cudaEventRecord(g.ev_cold[h], g.stream));
        return ORCHKV_OK;
    };
    if (n_chunks) {
        rc = gather(0);
        if (rc) return rc;
    }
    for (size_t c = 0; c < n_chunks; c++) {
        const size_t c0 = c * chunk, h = c % 2;
        const uint32_t k = (uint32_t)std::min<size_t>(chunk, io.size() - c0);
        OKV_CUDA_TRY(cudaEventSynchronize(g.ev_cold[h]));
        if (c + 1 < n_chunks) {                  // its half was written in the previous iteration
            rc = gather(c + 1);
            if (rc) return rc;
        }
        // write chunk c: consecutive file offsets in one pwritev each, the
        // runs spread over the IO workers
        std::vector<off_t> offs(k);
        std::vector<char *> bufs(k);
        for (uint32_t j = 0; j < k; j++) {
            offs[j] = io[c0 + j].off;
            bufs[j] = g.h_cold + (h * (size_t)chunk + j) * slab;
        }
        std::vector<iovec> iov;
        std::vector<IoRun> runs;
        plan_runs(offs, bufs, slab, iov, runs);
        if (!io_runs(true, ctx->fd, iov, runs)) {
            cudaStreamSynchronize(g.stream);      // the next gather may still write its half
            return ORCHKV_ERR_IO;
        }
    }
    rc = storage_commit(e, 2);
    if (rc) return rc;
    g.storage_writes += e.size();
    g.storage_bytes_written += e.size() * slab;
    if (result) { result[0] = (uint32_t)e.size(); result[1] = n - (uint32_t)e.size(); }
    return ORCHKV_OK;
}

int orchkv_block_id_table(kv_request_ctx_t *const *ctxs, uint32_t n, uint32_t row_len,
                          uint32_t *out)
{
    OKV_RANGE("orchkv_block_id_table");
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (!out || row_len == 0) return ORCHKV_ERR_INVALID;
    uint32_t L, H, mbph;
    int rc = upload_regions(ctxs, n, &L, &H, &mbph);
    if (rc) return rc;
    return launch_id_table(g.p, g.regions_dev, n, L, H, mbph, row_len, out, g.stream);
}

int orchkv_block_info(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi,
                      uint64_t *block_id, int *tier, uint32_t *slab, int *state,
                      uint32_t *token_count)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    const int rc = compat(ctx, OP_INFO, l, h, bi, 0);
    if (rc) return rc;
    const CompatResult &r = *g.res;
    if (block_id) *block_id = r.id;
    if (tier) *tier = (int)loc_tier(r.loc);
    if (slab) *slab = loc_slab(r.loc);
    if (state) *state = (int)r.state;
    if (token_count) *token_count = r.tok;
    return ORCHKV_OK;
}

int orchkv_set_block_flags(kv_request_ctx_t *ctx, uint32_t l, uint32_t h, uint32_t bi,
                           uint8_t flags)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    return compat(ctx, OP_SET_FLAGS, l, h, bi, flags);
}

int orchkv_read_pool(int which, uint32_t *stack_out, uint32_t *top_out)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (which < 0 || which > 2) return ORCHKV_ERR_INVALID;
    OKV_CUDA_TRY(cudaMemcpyAsync(g.h_ctr, g.p.ctr, sizeof(PoolCounters), cudaMemcpyDeviceToHost, g.stream));
    const uint32_t total = which == 0 ? g.p.g_total : which == 1 ? g.p.d_total : g.p.max_blocks;
    const uint32_t *stack = which == 0 ? g.p.g_stack : which == 1 ? g.p.d_stack : g.p.id_stack;
    if (stack_out)
        OKV_CUDA_TRY(cudaMemcpyAsync(stack_out, stack, (size_t)total * 4, cudaMemcpyDeviceToHost,
                                     g.stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    if (top_out)
        *top_out = which == 0 ? g.h_ctr->g_top : which == 1 ? g.h_ctr->d_top : g.h_ctr->id_top;
    return ORCHKV_OK;
}

int orchkv_read_block_locs(uint32_t *loc_out, uint8_t *state_out)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (loc_out)
        OKV_CUDA_TRY(cudaMemcpyAsync(loc_out, g.p.loc, (size_t)g.p.max_blocks * 4,
                                     cudaMemcpyDeviceToHost, g.stream));
    if (state_out)
        OKV_CUDA_TRY(cudaMemcpyAsync(state_out, g.p.state, g.p.max_blocks,
                                     cudaMemcpyDeviceToHost, g.stream));
    OKV_CUDA_TRY(cudaStreamSynchronize(g.stream));
    return ORCHKV_OK;
}

int orchkv_block_checksums(const uint32_t *ids, uint32_t n, unsigned long long *out,
                           uint8_t *tier_out)
{
    std::lock_guard<std::recursive_mutex> lk(g.mu);
    if (!g.inited) return ORCHKV_ERR_INIT;
    if (n && (!ids || !out)) return ORCHKV_ERR_INVALID;
    if (g.p.slab % 16) return ORCHKV_ERR_INVALID;     // the kernel reads 16-byte words
    return launch_block_checksums(g.p, ids, n, out, tier_out, g.stream);
}

uint32_t orchkv_max_blocks(void) { return g.inited ? g.p.max_blocks : 0; }

/* Number of CUDA kernel launches this library has issued since it loaded. */
unsigned long long orchkv_kernel_launches(void) { return launch_count(); }
void *orchkv_gpu_pool_base(void) { return g.inited ? g.p.gpu_base : nullptr; }
void *orchkv_dram_pool_base(void) { return g.inited ? g.p.dram_base : nullptr; }

}  // extern "C"
