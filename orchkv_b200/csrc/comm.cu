// comm.cu — NCCL communicator for the multi-GPU threshold exchange.
//
// The KV pool is sharded by KV head, one rank per GPU.  Scoring, packing and
// migration stay local; the only exchange is inside the selection: the
// per-pass key histograms are summed across ranks (ncclAllReduce, 16 KB) and
// the per-rank counts of boundary ties are gathered (ncclAllGather, 4 B per
// rank), so every rank evicts its share of the global coldest-k.
//
// NCCL is loaded with dlopen (the libnccl.so.2 that torch already loaded, if
// any), so the library has no link-time NCCL dependency.  Communicators are
// created non-blocking and every wait is bounded by a deadline, after which
// the communicator is aborted and an error returned.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>
#include <time.h>

#include <string>

#include "kernels.h"
#include "orchkv/tiered_manager.h"
#include "tm_internal.h"

namespace {

struct Nccl {
    void *h = nullptr;
    decltype(&ncclGetUniqueId) getUniqueId = nullptr;
    decltype(&ncclCommInitRankConfig) initRankConfig = nullptr;
    decltype(&ncclCommGetAsyncError) getAsyncError = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclAllReduce) allReduce = nullptr;
    decltype(&ncclAllGather) allGather = nullptr;
    decltype(&ncclGetErrorString) errStr = nullptr;
};

Nccl nccl;

bool load_nccl()
{
    if (nccl.h) return true;
    const char *names[] = {"libnccl.so.2", "libnccl.so"};
    for (const char *n : names) {
        nccl.h = dlopen(n, RTLD_NOW | RTLD_NOLOAD);
        if (nccl.h) break;
    }
    if (!nccl.h) {
        const char *env = getenv("ORCHKV_NCCL_LIB");
        if (env) nccl.h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
    }
    if (!nccl.h) nccl.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!nccl.h) return false;
#define OKV_SYM(f, n) nccl.f = (decltype(nccl.f))dlsym(nccl.h, n)
    OKV_SYM(getUniqueId, "ncclGetUniqueId");
    OKV_SYM(initRankConfig, "ncclCommInitRankConfig");
    OKV_SYM(getAsyncError, "ncclCommGetAsyncError");
    OKV_SYM(abort, "ncclCommAbort");
    OKV_SYM(destroy, "ncclCommDestroy");
    OKV_SYM(allReduce, "ncclAllReduce");
    OKV_SYM(allGather, "ncclAllGather");
    OKV_SYM(errStr, "ncclGetErrorString");
#undef OKV_SYM
    return nccl.getUniqueId && nccl.initRankConfig && nccl.getAsyncError && nccl.abort &&
           nccl.destroy && nccl.allReduce && nccl.allGather;
}

double now_s()
{
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + ts.tv_nsec * 1e-9;
}

constexpr int kTimedExchanges = 64;

struct Comm {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    double timeout = 30.0;
    bool broken = false;
    // device time of the exchanges since the last read: events around each
    // NCCL call on its stream (the first kTimedExchanges of them)
    cudaEvent_t ev[2 * kTimedExchanges] = {};
    uint32_t n_timed = 0, n_calls = 0;
};

void time_begin(Comm *c, cudaStream_t s)
{
    if (c->n_timed >= (uint32_t)kTimedExchanges) return;
    cudaEvent_t &e = c->ev[2 * c->n_timed];
    if (!e && cudaEventCreate(&e) != cudaSuccess) { e = nullptr; return; }
    cudaEventRecord(e, s);
}

void time_end(Comm *c, cudaStream_t s)
{
    c->n_calls++;
    if (c->n_timed >= (uint32_t)kTimedExchanges || !c->ev[2 * c->n_timed]) return;
    cudaEvent_t &e = c->ev[2 * c->n_timed + 1];
    if (!e && cudaEventCreate(&e) != cudaSuccess) { e = nullptr; return; }
    cudaEventRecord(e, s);
    c->n_timed++;
}

// Wait until a non-blocking NCCL call has been accepted; abort on timeout.
int settle(Comm *c, ncclResult_t r)
{
    if (r != ncclSuccess && r != ncclInProgress) {
        fprintf(stderr, "[orchkv] NCCL error: %s\n", nccl.errStr ? nccl.errStr(r) : "?");
        c->broken = true;
        return ORCHKV_ERR_CUDA;
    }
    const double deadline = now_s() + c->timeout;
    ncclResult_t st = r;
    while (st == ncclInProgress) {
        if (nccl.getAsyncError(c->comm, &st) != ncclSuccess) { st = ncclSystemError; break; }
        if (st == ncclInProgress && now_s() > deadline) {
            fprintf(stderr, "[orchkv] NCCL wait exceeded %.1f s; aborting communicator\n", c->timeout);
            nccl.abort(c->comm);
            c->comm = nullptr;
            c->broken = true;
            return ORCHKV_ERR_CUDA;
        }
    }
    if (st != ncclSuccess) {
        fprintf(stderr, "[orchkv] NCCL async error: %s\n", nccl.errStr ? nccl.errStr(st) : "?");
        c->broken = true;
        return ORCHKV_ERR_CUDA;
    }
    return ORCHKV_OK;
}

int reduce_hist(const uint32_t *local, uint32_t *global, uint32_t n, cudaStream_t s, void *ctx)
{
    Comm *c = (Comm *)ctx;
    if (!c || c->broken || !c->comm) return ORCHKV_ERR_CUDA;
    time_begin(c, s);
    const int rc = settle(c, nccl.allReduce(local, global, n, ncclUint32, ncclSum, c->comm, s));
    time_end(c, s);
    return rc;
}

int gather_one(const uint32_t *one, uint32_t *all, cudaStream_t s, void *ctx)
{
    Comm *c = (Comm *)ctx;
    if (!c || c->broken || !c->comm) return ORCHKV_ERR_CUDA;
    time_begin(c, s);
    const int rc = settle(c, nccl.allGather(one, all, 1, ncclUint32, c->comm, s));
    time_end(c, s);
    return rc;
}

}  // namespace

extern "C" {

/* Fill `out` (128 bytes) with a new NCCL unique id (rank 0 calls this and
 * broadcasts the bytes).  Returns ORCHKV_ERR_INIT if NCCL cannot be loaded. */
int orchkv_comm_unique_id(unsigned char *out)
{
    if (!out) return ORCHKV_ERR_INVALID;
    if (!load_nccl()) return ORCHKV_ERR_INIT;
    ncclUniqueId id;
    if (nccl.getUniqueId(&id) != ncclSuccess) return ORCHKV_ERR_CUDA;
    memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return ORCHKV_OK;
}

/* Create this rank's communicator (non-blocking init, bounded by timeout_s).
 * The current CUDA device must be this rank's GPU.  NULL on failure. */
void *orchkv_comm_create(int rank, int world, const unsigned char *id_bytes, double timeout_s)
{
    if (!id_bytes || world < 1 || rank < 0 || rank >= world) return nullptr;
    if (!load_nccl()) return nullptr;
    Comm *c = new Comm();
    c->rank = rank;
    c->world = world;
    c->timeout = timeout_s > 0 ? timeout_s : 30.0;
    ncclUniqueId id;
    memcpy(id.internal, id_bytes, NCCL_UNIQUE_ID_BYTES);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = nccl.initRankConfig(&c->comm, world, id, rank, &cfg);
    if (settle(c, r) != ORCHKV_OK) {
        if (c->comm) nccl.abort(c->comm);
        delete c;
        return nullptr;
    }
    return c;
}

/* Device time spent in this communicator's exchanges (histogram all-reduces
 * and tie all-gathers, each timed on its stream, waits for slower ranks
 * included) since the previous call, and how many there were; then starts
 * over.  Synchronises on the timed events. */
int orchkv_comm_exchange_time(void *h, float *ms, uint32_t *calls)
{
    Comm *c = (Comm *)h;
    if (!c) return ORCHKV_ERR_INVALID;
    float total = 0.f;
    for (uint32_t i = 0; i < c->n_timed; i++) {
        float x = 0.f;
        if (cudaEventSynchronize(c->ev[2 * i + 1]) != cudaSuccess ||
            cudaEventElapsedTime(&x, c->ev[2 * i], c->ev[2 * i + 1]) != cudaSuccess)
            return ORCHKV_ERR_CUDA;
        total += x;
    }
    if (ms) *ms = total;
    if (calls) *calls = c->n_calls;
    c->n_timed = 0;
    c->n_calls = 0;
    return ORCHKV_OK;
}

int orchkv_comm_destroy(void *h)
{
    Comm *c = (Comm *)h;
    if (!c) return ORCHKV_ERR_INVALID;
    for (auto &e : c->ev) if (e) cudaEventDestroy(e);
    if (c->comm) {
        if (c->broken) nccl.abort(c->comm);
        else nccl.destroy(c->comm);
    }
    delete c;
    return ORCHKV_OK;
}

/* Sum-all-reduce of n uint32 on `stream` (also used by tests). */
int orchkv_comm_allreduce_u32(void *h, const uint32_t *send, uint32_t *recv, uint32_t n,
                              void *stream)
{
    return reduce_hist(send, recv, n, (cudaStream_t)stream, h);
}

/* Route the manager's selections through the communicator: k and fractions
 * then refer to the union of all ranks' blocks, ties split by rank order.
 * A one-rank communicator takes the same path (its exchanges are local
 * copies and the picks those of a detached manager).  NULL detaches. */
int tm_set_comm(tiered_manager_t *m, void *h)
{
    TmImpl *t = tm_impl(m);
    if (!t) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> g(t->mu);
    Comm *c = (Comm *)h;
    if (c && c->world > kMaxSelectRanks) return ORCHKV_ERR_INVALID;   // tie gather room
    if (!c) {
        t->comm_reduce = nullptr;
        t->comm_gather = nullptr;
        t->comm_ctx = nullptr;
        t->comm_rank = 0;
        t->comm_world = 1;
        return ORCHKV_OK;
    }
    t->comm_reduce = reduce_hist;
    t->comm_gather = gather_one;
    t->comm_ctx = c;
    t->comm_rank = c->rank;
    t->comm_world = c->world;
    return ORCHKV_OK;
}

}  // extern "C"
