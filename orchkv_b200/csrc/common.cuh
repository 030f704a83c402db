// common.cuh — device-side definitions shared by the orchkv B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <nvtx3/nvToolsExt.h>

#include "orchkv/kv_types.h"

namespace okv {

constexpr uint32_t kNoBlock = 0xFFFFFFFFu;
constexpr unsigned long long kStepNever = ~0ull;
constexpr uint32_t kKeyInvalid = 0xFFFFFFFFu;   // ineligible in a selection
constexpr uint32_t kLocTierShift = 29;
constexpr uint32_t kLocSlabMask = 0x1FFFFFFFu;
constexpr int kDecayTable = 512;                  // hotcold_classifier.h:63

__host__ __device__ inline uint32_t make_loc(uint32_t tier, uint32_t slab)
{
    return (tier << kLocTierShift) | (slab & kLocSlabMask);
}
__host__ __device__ inline uint32_t loc_tier(uint32_t w) { return w >> kLocTierShift; }
__host__ __device__ inline uint32_t loc_slab(uint32_t w) { return w & kLocSlabMask; }

// Orderable key of a float: ascending key == ascending value; -0 folded on
// +0 (equal under the callers' comparison sort), NaN after all numbers.
__host__ __device__ inline uint32_t orderable(float f)
{
    if (f != f) return 0xFFFFFFFEu;
    if (f == 0.0f) f = 0.0f;
#ifdef __CUDA_ARCH__
    uint32_t u = __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
#endif
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Per-slot scheduler state (tracker + classifier + selector view), one
// structure-of-arrays per manager, indexed by slot = block_id & mask.
struct SchedDev {
    float *sum, *mx, *ema, *hot;
    uint32_t *hits;
    unsigned long long *last;
    uint8_t *tact;     // tracker slot active
    uint8_t *cact;     // classifier slot active
    uint8_t *cflags;   // flags captured at registration (ATTN_SINK check)
    uint8_t *heat;
    uint8_t *tier;     // StorageTier of the block as the selector sees it
    uint8_t *bflags;   // live block flags (PIN check)
    uint8_t *bstate;   // KVBlockState (MIGRATING check)
    uint32_t *key;     // selection scratch
    const float *table;
    uint32_t cap, mask;
};

struct SchedParams {
    float lambda, one_minus, alpha, beta, gamma, th_hot, th_warm;
    unsigned long long step;
};

// Counters produced by the classification sweep.
struct ClassCounts {
    uint32_t n_hot, n_warm, n_cold, n_sink;
};

// Host-side count of kernel launches issued by this library (every launcher
// adds the launches it enqueues); exported as orchkv_kernel_launches().
void note_launches(unsigned n);
unsigned long long launch_count();

// ---- small block-wide helpers ------------------------------------------------

__device__ inline uint32_t warp_incl_scan(uint32_t v)
{
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t n = __shfl_up_sync(0xFFFFFFFFu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Exclusive scan across the block (blockDim.x multiple of 32, <= 1024).
// `tmp` must hold 33 uint32.  Returns the exclusive prefix; *total gets the sum.
__device__ inline uint32_t block_excl_scan(uint32_t v, uint32_t *tmp, uint32_t *total)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    uint32_t inc = warp_incl_scan(v);
    if (lane == 31) tmp[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        uint32_t w = lane < nw ? tmp[lane] : 0;
        uint32_t wi = warp_incl_scan(w);
        if (lane < nw) tmp[lane] = wi - w;
        if (lane == nw - 1) tmp[32] = wi;
    }
    __syncthreads();
    uint32_t r = tmp[wid] + inc - v;
    if (total) *total = tmp[32];
    __syncthreads();
    return r;
}

// A named range on the profiler timeline (Nsight Systems, ncu's NVTX
// filters) for the duration of a host call; a no-op unless a tool is attached.
struct OkvRange {
    explicit OkvRange(const char *name) { nvtxRangePushA(name); }
    ~OkvRange() { nvtxRangePop(); }
};

}  // namespace okv

#define OKV_RANGE(name) okv::OkvRange okv_range_(name)

#define OKV_CUDA_TRY(call)                                                      \
    do {                                                                        \
        cudaError_t _e = (call);                                                \
        if (_e != cudaSuccess) {                                                \
            fprintf(stderr, "[orchkv] CUDA error %d (%s) at %s:%d\n", (int)_e,  \
                    cudaGetErrorString(_e), __FILE__, __LINE__);                \
            return ORCHKV_ERR_CUDA;                                             \
        }                                                                       \
    } while (0)
