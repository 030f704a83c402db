// static_select.cu — coldest-k selection that allocates no memory.
//
// Some callers cannot call cudaMalloc while they run: serving engines that
// reserve the device's memory for their own allocator at start-up (a stray
// cudaMalloc then fails or fragments that reservation), and real-time paths
// that must not take the CUDA allocator's locks.  For them this entry point
// runs the same radix selection as tm_select_victims over a caller-provided
// value array, with every scratch word (keys, histograms, selection state,
// compaction tiles) in the file-scope device array below.  The caller still
// passes the inputs and the outputs.
#include <cuda.h>

#include <mutex>

#include "kernels.h"
#include "orchkv/tiered_manager.h"

namespace {

constexpr uint32_t kNoAllocMaxN = 1u << 20;                 // 1,048,576 values
constexpr uint32_t kNoAllocTiles = (kNoAllocMaxN + 4095) / 4096;
constexpr size_t kHistWords = 4096 + 16;
constexpr size_t kScratchWords = kNoAllocMaxN + 2 * kHistWords + 16 + 4 * (size_t)kNoAllocTiles;

// ~4.1 MB per GPU that loads the library, held until the process exits.
static __device__ __align__(256) uint32_t g_noalloc_scratch[kScratchWords];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint32_t *g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};
typedef CUresult (*CtxGetCurrentFn)(CUcontext *);
CtxGetCurrentFn g_ctx_current = nullptr;

// The context the calling thread runs in on this device (a thread-local read
// in the driver), so an address looked up in a context that has since been
// destroyed -- cudaDeviceReset -- is not reused.
CUcontext current_context()
{
    if (!g_ctx_current) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        g_ctx_current = (CtxGetCurrentFn)fn;
    }
    CUcontext c = nullptr;
    return g_ctx_current(&c) == CUDA_SUCCESS ? c : nullptr;
}

// The array's name is only a host-side stand-in: its device address is looked
// up once per device (and again only if that device's context was replaced),
// with that device current.
int scratch_for_current_device(uint32_t **out)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ORCHKV_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return ORCHKV_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_mu);
    // null until this thread's first runtime call that needs the device;
    // the lookup below makes the context current
    const CUcontext ctx = current_context();
    if (!g_scratch_addr[dev] || !ctx || ctx != g_scratch_ctx[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            fprintf(stderr, "[orchkv] cudaGetSymbolAddress(static selection scratch) failed: %s\n",
                    cudaGetErrorString(e));
            return ORCHKV_ERR_CUDA;
        }
        g_scratch_addr[dev] = static_cast<uint32_t *>(p);
        g_scratch_ctx[dev] = current_context();
    }
    *out = g_scratch_addr[dev];
    return ORCHKV_OK;
}

}  // namespace

extern "C" int orchkv_select_coldest_noalloc(const float *values, const uint8_t *eligible,
                                             uint32_t n, uint32_t k, uint32_t *out_ids,
                                             uint32_t *out_count, void *stream)
{
    if (n > kNoAllocMaxN) {
        fprintf(stderr, "[orchkv] orchkv_select_coldest_noalloc: n = %u exceeds the static "
                        "scratch capacity of %u values\n", n, kNoAllocMaxN);
        return ORCHKV_ERR_INVALID;
    }
    if (!out_count || (n > 0 && (!values || !eligible || (k > 0 && !out_ids))))
        return ORCHKV_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (n == 0 || k == 0) {
        OKV_CUDA_TRY(cudaMemsetAsync(out_count, 0, sizeof(uint32_t), s));
        return ORCHKV_OK;
    }
    uint32_t *scratch = nullptr;
    int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;

    okv::SchedDev d;
    memset(&d, 0, sizeof(d));
    d.hot = const_cast<float *>(values);
    d.tact = const_cast<uint8_t *>(eligible);
    d.key = scratch;
    d.cap = n;
    d.mask = 0xFFFFFFFFu;

    okv::SelectScratch sc;
    sc.hist_local = scratch + kNoAllocMaxN;
    sc.hist_global = sc.hist_local + kHistWords;
    sc.state = sc.hist_global + kHistWords;
    sc.tile_counts = sc.state + 16;
    sc.tile_offsets = sc.tile_counts + 2 * kNoAllocTiles;
    sc.max_tiles = kNoAllocTiles;

    okv::SelectArgs a;
    memset(&a, 0, sizeof(a));
    a.mode = okv::kSelectExternal;
    a.k = k;
    a.frac = -1.0f;
    a.max_out = k;
    a.out_ids = out_ids;
    a.out_count = out_count;
    a.world = 1;
    return okv::launch_select(d, sc, a, s);
}
