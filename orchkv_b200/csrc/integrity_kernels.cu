// integrity_kernels.cu — per-block checksums of slab contents on the device.
//
// The reference checks migrated bytes by writing `seed ^ i` words into a slab
// and comparing them word by word after the round trip
// (test/test_gpu_dram.cu:40-55,151-243).  At the path's real sizes (millions
// of 8-32 KB slabs) copying every slab out to compare it is the slow part, so
// a block's bytes are reduced where they live to one 64-bit word:
//
//     c = sum_i x_i * m_i  (mod 2^64),   m_i = mix64(i) | 1
//
// x_i is the i-th little-endian 64-bit word of the slab and mix64 the
// splitmix64 output function (Steele, Lea, Flood, "Fast splittable
// pseudorandom number generators", OOPSLA 2014).  Every m_i is odd, so a
// change of any single word always changes c, and words that trade places
// change it unless their multipliers happen to agree.  A host can recompute c
// from the same definition (numpy wraps uint64 products and sums the same way).
#include "kernels.h"
#include "pool.h"

namespace okv {

namespace {

__device__ __forceinline__ unsigned long long mix64(unsigned long long z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

constexpr int kSumWarps = 8;

// One warp per listed block: lanes stride the slab in 16-byte loads (two
// words each), products are summed per lane and then across the warp.
// Blocks that are neither in HBM nor in the DRAM tier (storage, unknown id)
// get 0 and tier 7.
__global__ void __launch_bounds__(kSumWarps * 32)
block_checksum_kernel(PoolDev p, const uint32_t *__restrict__ ids, uint32_t n,
                      unsigned long long *__restrict__ out, uint8_t *__restrict__ tier_out)
{
    const uint32_t w = blockIdx.x * kSumWarps + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= n) return;
    const uint32_t id = ids[w];
    uint32_t tier = 7;
    const char *src = nullptr;
    if (id < p.max_blocks) {
        const uint32_t loc = p.loc[id];
        tier = loc_tier(loc);
        const uint32_t slab = loc_slab(loc);
        if (tier == TIER_GPU_HBM && slab < p.g_total) src = p.gpu_base + (size_t)slab * p.slab;
        else if (tier == TIER_HOST_DRAM && slab < p.d_total) src = p.dram_base + (size_t)slab * p.slab;
        else tier = 7;
    }
    unsigned long long acc = 0;
    if (src) {
        const ulonglong2 *v = reinterpret_cast<const ulonglong2 *>(src);
        const uint32_t nv = (uint32_t)(p.slab / 16);
        for (uint32_t j = lane; j < nv; j += 32) {
            const ulonglong2 x = v[j];
            acc += x.x * (mix64(2ull * j) | 1ull);
            acc += x.y * (mix64(2ull * j + 1) | 1ull);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) {
        out[w] = acc;
        if (tier_out) tier_out[w] = (uint8_t)tier;
    }
}

}  // namespace

int launch_block_checksums(const PoolDev &p, const uint32_t *ids, uint32_t n,
                           unsigned long long *out, uint8_t *tier_out, cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    const unsigned grid = (n + kSumWarps - 1) / kSumWarps;
    block_checksum_kernel<<<grid, kSumWarps * 32, 0, s>>>(p, ids, n, out, tier_out);
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

}  // namespace okv
