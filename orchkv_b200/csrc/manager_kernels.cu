// manager_kernels.cu — data movement for callers that keep their own
// contiguous per-layer KV buffers (the Python managers' persistent buffers,
// python/orchkv/fast_kvcache_manager.py:79-88): token blocks of all layers
// copied to or from a packed store in one launch, instead of one .cpu() /
// .to("cuda") pair per (block, layer) (fast_kvcache_manager.py:204-219,
// 324-338).
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"
#include "orchkv/orchkv_api.h"

namespace okv {
namespace {

constexpr uint32_t kMaxBufs = 1024;   // 8 KB of kernel parameters

struct BufTable {
    char *p[kMaxBufs];
};

// One warp per (block j, buffer, head) chunk: rows [0, n) of
// block_tokens x row_bytes, 16-byte lanes.
__global__ void __launch_bounds__(256)
token_block_copy_kernel(const __grid_constant__ BufTable bufs, uint32_t n_bufs, uint32_t n_heads,
                        unsigned long long head_stride, uint32_t row_bytes,
                        uint32_t block_tokens, uint32_t n_tokens, const uint32_t *blocks,
                        uint32_t n_blocks, char *store, const uint32_t *slots, int dir)
{
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long chunks = (unsigned long long)n_blocks * n_bufs * n_heads;
    const unsigned long long warp0 = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    const unsigned long long chunk_bytes = (unsigned long long)block_tokens * row_bytes;
    for (unsigned long long c = warp0; c < chunks; c += nwarps) {
        const uint32_t h = (uint32_t)(c % n_heads);
        const uint32_t bi = (uint32_t)((c / n_heads) % n_bufs);
        const uint32_t j = (uint32_t)(c / ((unsigned long long)n_heads * n_bufs));
        const uint32_t b = blocks[j];
        const unsigned long long t0 = (unsigned long long)b * block_tokens;
        if (t0 >= n_tokens) continue;
        const unsigned long long rows = n_tokens - t0 < block_tokens ? n_tokens - t0 : block_tokens;
        char *buf = bufs.p[bi] + h * head_stride + t0 * row_bytes;
        const unsigned long long slot = slots ? slots[j] : j;
        char *st = store + ((slot * n_bufs + bi) * n_heads + h) * chunk_bytes;
        const uint4 *s = reinterpret_cast<const uint4 *>(dir == 0 ? buf : st);
        uint4 *d = reinterpret_cast<uint4 *>(dir == 0 ? st : buf);
        const unsigned long long nvec = rows * row_bytes / 16;
        unsigned long long i = lane;
        for (; i + 3 * 32 < nvec; i += 4 * 32) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) v[u] = s[i + u * 32];
#pragma unroll
            for (int u = 0; u < 4; u++) d[i + u * 32] = v[u];
        }
        for (; i < nvec; i += 32) d[i] = s[i];
    }
}

// A pointer kernels can address: device memory as is, pinned host memory
// through its mapping; nullptr for pageable memory.
char *kernel_ptr(void *p)
{
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return (char *)p;
    if (a.type == cudaMemoryTypeHost && a.devicePointer) return (char *)a.devicePointer;
    return nullptr;
}

}  // namespace
}  // namespace okv

extern "C" int orchkv_copy_token_blocks(void *const *bufs, uint32_t n_bufs, uint32_t n_heads,
                                        uint64_t head_stride_bytes, uint32_t row_bytes,
                                        uint32_t block_tokens, uint32_t n_tokens,
                                        const uint32_t *blocks, uint32_t n_blocks, void *store,
                                        const uint32_t *store_slots, int dir, void *stream)
{
    using namespace okv;
    if (n_blocks == 0) return ORCHKV_OK;
    if (!bufs || !blocks || !store || n_bufs == 0 || n_bufs > kMaxBufs || n_heads == 0 ||
        block_tokens == 0 || (dir != 0 && dir != 1))
        return ORCHKV_ERR_INVALID;
    if (row_bytes == 0 || row_bytes % 16 || head_stride_bytes % 16) return ORCHKV_ERR_INVALID;
    BufTable t;
    for (uint32_t i = 0; i < n_bufs; i++) {
        t.p[i] = bufs[i] ? kernel_ptr(bufs[i]) : nullptr;
        if (!t.p[i] || (uintptr_t)t.p[i] % 16) return ORCHKV_ERR_INVALID;
    }
    char *st = kernel_ptr(store);
    if (!st || (uintptr_t)st % 16 || !kernel_ptr((void *)blocks)) return ORCHKV_ERR_INVALID;
    if (store_slots && !kernel_ptr((void *)store_slots)) return ORCHKV_ERR_INVALID;
    const unsigned long long chunks = (unsigned long long)n_blocks * n_bufs * n_heads;
    unsigned grid = (unsigned)((chunks + 7) / 8);
    if (grid > 148 * 16) grid = 148 * 16;
    token_block_copy_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        t, n_bufs, n_heads, head_stride_bytes, row_bytes, block_tokens, n_tokens, blocks,
        n_blocks, st, store_slots, dir);
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}
