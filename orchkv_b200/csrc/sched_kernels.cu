// sched_kernels.cu — attention scoring (K1) and the tracker/classifier sweep
// (K2) of the orchkv B200 scheduler.
//
// K1 replaces the managers' per-block torch reduction + pybind report loop
// (python/orchkv/fast_kvcache_manager.py:221-235) and attn_tracker_update
// (src/scheduler/attention_tracker.c:27-33,75-118).  K2 replaces the
// O(capacity) host sweeps attn_tracker_step_done
// (src/scheduler/attention_tracker.c:120-150) and hcc_update_all
// (src/scheduler/hotcold_classifier.c:69-83,161-185).
//
// Float semantics: every product and sum in K2 uses __fmul_rn / __fadd_rn /
// __fdiv_rn so no FMA is formed and each operation rounds exactly as the
// reference's single-precision host code; the recency table is built on the
// host with libm expf (as the reference does) and only read here.
#include <atomic>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "kernels.h"

namespace okv {

static std::atomic<unsigned long long> g_launches{0};
void note_launches(unsigned n) { g_launches += n; }
unsigned long long launch_count() { return g_launches.load(); }

// ---------------------------------------------------------------------------
// K1: per-block attention mass
// ---------------------------------------------------------------------------

__device__ __forceinline__ float4 ld_stream(const float4 *p)
{
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void record_mass(const SchedDev &d, uint32_t id, float w,
                                            unsigned long long step)
{
    if (id == kNoBlock) return;
    const uint32_t s = id & d.mask;
    if (!d.tact[s]) return;                     // inactive slots ignore reports
    d.sum[s] = __fadd_rn(d.sum[s], w);
    if (w > d.mx[s]) d.mx[s] = w;
    d.last[s] = step;
}

constexpr int kScoreWarps = 8;     // warps per CTA
constexpr int kScoreU = 4;         // float4 columns per lane per row: 512-token tiles

// One warp per tile (row r, KV head h, 512-token chunk).  Lane l of step u
// loads float4 column (chunk*128 + u*32 + l) of each of the G query-head rows
// of KV group h: every load instruction is one fully coalesced 512-byte line.
// Token blocks of tpb tokens cover tpb/4 consecutive lanes and are summed with
// xor-shuffles.  The tile's blocks are then spread over the lanes (block k of
// the tile to lane k % 32), whose tracker entries were fetched while the
// probability rows streamed in, so recording costs no extra round trip.
// A minimum of one resident CTA lets the compiler keep more loads in flight
// per warp (72 registers, 3 CTAs per SM): measured 9% faster than the
// default 52-register build at 4 CTAs per SM.
template <int LOG_LPB>
__global__ void __launch_bounds__(kScoreWarps * 32, 1)
score_vec_kernel(const float *__restrict__ probs, uint32_t Hq, uint32_t Hkv,
                 uint32_t T, uint32_t tpb, const uint32_t *__restrict__ lens,
                 const uint32_t *__restrict__ ids, uint32_t nb, uint32_t n_chunks,
                 unsigned long long n_tiles, SchedDev d, unsigned long long step,
                 ReportOrder o)
{
    constexpr int LPB = 1 << LOG_LPB;              // lanes per block in one step
    constexpr int BPU = 32 / LPB;                  // blocks per step
    constexpr int NBLK = kScoreU * BPU;            // blocks per tile
    constexpr int K = NBLK > 32 ? NBLK / 32 : 1;   // blocks recorded per lane
    const int lane = threadIdx.x & 31;
    const unsigned long long tile =
        (unsigned long long)blockIdx.x * kScoreWarps + (threadIdx.x >> 5);
    if (tile >= n_tiles) return;
    const uint32_t c = (uint32_t)(tile % n_chunks);
    const unsigned long long rh = tile / n_chunks;
    const uint32_t h = (uint32_t)(rh % Hkv);
    const unsigned long long r = rh / Hkv;
    const uint32_t G = Hq / Hkv;
    uint32_t len = lens ? lens[r] : T;
    if (len > T) len = T;
    const uint32_t T4 = T >> 2;
    const float4 *base = reinterpret_cast<const float4 *>(probs + (r * Hq + (unsigned long long)h * G) * T);
    const bool ordered = *o.flag == o.epoch;       // this call's ids alias: no direct records

    // block ids of the blocks this lane records
    uint32_t bid[K];
#pragma unroll
    for (int j = 0; j < K; j++) {
        const uint32_t k = (uint32_t)lane + 32u * j;
        const uint32_t b = c * NBLK + k;
        bid[j] = (k < (uint32_t)NBLK && b < nb && b * tpb < len) ? ids[rh * nb + b] : kNoBlock;
    }

    const uint32_t col0 = c * (32 * kScoreU) + lane;
    // row 0 of the group: its loads are issued first, then the tracker
    // entries are fetched under them
    float4 acc[kScoreU];
#pragma unroll
    for (int u = 0; u < kScoreU; u++) {
        const uint32_t col = col0 + u * 32;
        acc[u] = col < T4 ? ld_stream(base + col) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    uint8_t act[K];
    float old_sum[K], old_max[K];
#pragma unroll
    for (int j = 0; j < K; j++) {
        act[j] = 0; old_sum[j] = 0.f; old_max[j] = 0.f;
        if (bid[j] != kNoBlock) {
            const uint32_t sl = bid[j] & d.mask;
            act[j] = d.tact[sl];
            old_sum[j] = d.sum[sl];
            old_max[j] = d.mx[sl];
        }
    }
    // remaining rows in order g = 1, 2, ...
    for (uint32_t g = 1; g < G; g++) {
        const float4 *rg = base + (unsigned long long)g * T4;
        float4 a[kScoreU];
#pragma unroll
        for (int u = 0; u < kScoreU; u++) {
            const uint32_t col = col0 + u * 32;
            a[u] = col < T4 ? ld_stream(rg + col) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kScoreU; u++) {
            acc[u].x += a[u].x; acc[u].y += a[u].y;
            acc[u].z += a[u].z; acc[u].w += a[u].w;
        }
    }

    float part[kScoreU];
#pragma unroll
    for (int u = 0; u < kScoreU; u++) {
        const uint32_t t0 = (col0 + u * 32) * 4;
        // tokens at or beyond the row's valid length contribute nothing
        float4 a = acc[u];
        if (t0 + 0 >= len) a.x = 0.f;
        if (t0 + 1 >= len) a.y = 0.f;
        if (t0 + 2 >= len) a.z = 0.f;
        if (t0 + 3 >= len) a.w = 0.f;
        float sv = (a.x + a.y) + (a.z + a.w);
#pragma unroll
        for (int o = 1; o < LPB; o <<= 1) sv += __shfl_xor_sync(0xFFFFFFFFu, sv, o);
        part[u] = sv;                  // block (u, lane / LPB) total, on its lanes
    }
#pragma unroll
    for (int j = 0; j < K; j++) {
        const uint32_t k = (uint32_t)lane + 32u * j;
        const uint32_t uk = k / BPU;                 // step holding block k
        const int src = (int)((k % BPU) * LPB);      // a lane of block k in that step
        float w = 0.f;
#pragma unroll
        for (int u = 0; u < kScoreU; u++) {
            const float t = __shfl_sync(0xFFFFFFFFu, part[u], src);
            if (uk == (uint32_t)u) w = t;
        }
        if (ordered) {
            const uint32_t b = c * NBLK + k;
            if (k < (uint32_t)NBLK && b < nb) {
                o.ids_eff[rh * nb + b] = bid[j];
                o.mass[rh * nb + b] = w;
            }
        } else if (bid[j] != kNoBlock && act[j]) {
            const uint32_t sl = bid[j] & d.mask;
            d.sum[sl] = __fadd_rn(old_sum[j], w);
            if (w > old_max[j]) d.mx[sl] = w;
            d.last[sl] = step;
        }
    }
}

// Fallback for any geometry the vector kernel does not take (tpb not a power
// of two in [4,128], T not a multiple of 4, unaligned rows): one thread per
// (row, KV head, block), summing in the oracle's loop order.
__global__ void score_scalar_kernel(const float *__restrict__ probs, uint32_t Hq,
                                    uint32_t Hkv, uint32_t T, uint32_t tpb,
                                    const uint32_t *__restrict__ lens,
                                    const uint32_t *__restrict__ ids, uint32_t nb,
                                    unsigned long long n_items, SchedDev d,
                                    unsigned long long step, ReportOrder o)
{
    const unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_items) return;
    const bool ordered = *o.flag == o.epoch;
    const uint32_t b = (uint32_t)(i % nb);
    const unsigned long long rh = i / nb;
    const uint32_t h = (uint32_t)(rh % Hkv);
    const unsigned long long r = rh / Hkv;
    const uint32_t G = Hq / Hkv;
    uint32_t len = lens ? lens[r] : T;
    if (len > T) len = T;
    const uint32_t t0 = b * tpb;
    if (t0 >= len) {
        if (ordered) o.ids_eff[i] = kNoBlock;
        return;
    }
    uint32_t t1 = t0 + tpb;
    if (t1 > len) t1 = len;
    float acc = 0.0f;
    for (uint32_t g = 0; g < G; g++) {
        const float *row = probs + ((r * Hq) + (unsigned long long)h * G + g) * T;
        for (uint32_t t = t0; t < t1; t++) acc = __fadd_rn(acc, row[t]);
    }
    if (ordered) {
        o.ids_eff[i] = ids[i];
        o.mass[i] = acc;
    } else {
        record_mass(d, ids[i], acc, step);
    }
}

// ---------------------------------------------------------------------------
// Reports whose ids share tracker slots within one call
// ---------------------------------------------------------------------------

// Stamps each listed active slot with the call's epoch; a slot stamped twice
// means two entries would update it: the call then takes the ordered pass.
__global__ void alias_mark_kernel(const uint32_t *__restrict__ ids, uint32_t n, SchedDev d,
                                  ReportOrder o)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t id = ids[i];
    if (id == kNoBlock) return;
    const uint32_t s = id & d.mask;
    if (!d.tact[s]) return;                        // inactive slots ignore reports
    if (atomicExch(&o.mark[s], o.epoch) == o.epoch) *o.flag = o.epoch;
}

int launch_alias_mark(const uint32_t *ids, uint32_t n, const SchedDev &d, const ReportOrder &o,
                      cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    alias_mark_kernel<<<(n + 255) / 256, 256, 0, s>>>(ids, n, d, o);
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

constexpr int kOrderThreads = 1024;
constexpr unsigned kOrderCtas = 296;          // two 1024-thread CTAs on each of 148 SMs

// The ordered pass.  CTA c owns the slots with slot % gridDim.x == c and walks
// the whole list in chunks of 1024 entries; a chunk's owned entries are
// compacted in entry order into shared memory and applied by warp 0, 32 at a
// time: lanes holding the same slot are grouped (__match_any_sync) and the
// group's lowest lane adds their masses in lane order, so every slot sees its
// entries' additions in list order, exactly as that many single reports.
__global__ void __launch_bounds__(kOrderThreads)
report_ordered_kernel(const uint32_t *__restrict__ ids, const float *__restrict__ w, uint32_t n,
                      SchedDev d, unsigned long long step, ReportOrder o)
{
    if (*o.flag != o.epoch) return;
    __shared__ uint32_t s_slot[kOrderThreads];
    __shared__ float s_w[kOrderThreads];
    __shared__ uint32_t tmp[33];
    const uint32_t owner = blockIdx.x, owners = gridDim.x;
    const int lane = threadIdx.x & 31;
    for (uint32_t base = 0; base < n; base += kOrderThreads) {
        const uint32_t i = base + threadIdx.x;
        const uint32_t id = i < n ? ids[i] : kNoBlock;
        const uint32_t slot = id & d.mask;
        const bool own = id != kNoBlock && slot % owners == owner;
        uint32_t total;
        const uint32_t pos = block_excl_scan(own ? 1u : 0u, tmp, &total);
        if (own) {
            s_slot[pos] = slot;
            s_w[pos] = w[i];
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            for (uint32_t q = 0; q < total; q += 32) {
                const uint32_t j = q + lane;
                const bool has = j < total;
                const uint32_t sl = has ? s_slot[j] : 0xFFFFFFFFu;
                const unsigned peers = __match_any_sync(0xFFFFFFFFu, sl);
                if (has && lane == __ffs(peers) - 1 && d.tact[sl]) {
                    float sum = d.sum[sl], mx = d.mx[sl];
                    for (unsigned m = peers; m; m &= m - 1) {
                        const float x = s_w[q + __ffs(m) - 1];
                        sum = __fadd_rn(sum, x);
                        if (x > mx) mx = x;
                    }
                    d.sum[sl] = sum;
                    d.mx[sl] = mx;
                    d.last[sl] = step;
                }
                __syncwarp();
            }
        }
        __syncthreads();
    }
}

int launch_report_ordered(const uint32_t *ids, const float *w, uint32_t n, const SchedDev &d,
                          unsigned long long step, const ReportOrder &o, cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    report_ordered_kernel<<<kOrderCtas, kOrderThreads, 0, s>>>(ids, w, n, d, step, o);
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

int launch_score(const float *probs, uint32_t R, uint32_t Hq, uint32_t Hkv,
                 uint32_t T, uint32_t tpb, const uint32_t *lens,
                 const uint32_t *ids, const SchedDev &d, unsigned long long step,
                 const ReportOrder &o, cudaStream_t s)
{
    if (!probs || !ids || R == 0 || Hq == 0 || Hkv == 0 || T == 0 || tpb == 0 ||
        Hq % Hkv != 0)
        return ORCHKV_ERR_INVALID;
    const uint32_t nb = (T + tpb - 1) / tpb;
    const bool pow2 = (tpb & (tpb - 1)) == 0;
    const bool vec_ok = pow2 && tpb >= 4 && tpb <= 128 && (T % 4) == 0 &&
                        ((uintptr_t)probs % 16) == 0;
    if (vec_ok) {
        const uint32_t n_chunks = (T + 128 * kScoreU - 1) / (128 * kScoreU);
        const unsigned long long n_tiles = (unsigned long long)R * Hkv * n_chunks;
        const unsigned long long grid = (n_tiles + kScoreWarps - 1) / kScoreWarps;
        const int log_lpb = __builtin_ctz(tpb / 4);
#define OKV_SCORE_CASE(L)                                                              \
    case L:                                                                            \
        score_vec_kernel<L><<<(unsigned)grid, kScoreWarps * 32, 0, s>>>(               \
            probs, Hq, Hkv, T, tpb, lens, ids, nb, n_chunks, n_tiles, d, step, o);             \
        note_launches(1);                                                              \
        break;
        switch (log_lpb) {
            OKV_SCORE_CASE(0) OKV_SCORE_CASE(1) OKV_SCORE_CASE(2)
            OKV_SCORE_CASE(3) OKV_SCORE_CASE(4) OKV_SCORE_CASE(5)
            default: return ORCHKV_ERR_INVALID;
        }
#undef OKV_SCORE_CASE
    } else {
        const unsigned long long n_items = (unsigned long long)R * Hkv * nb;
        const unsigned grid = (unsigned)((n_items + 255) / 256);
        score_scalar_kernel<<<grid, 256, 0, s>>>(probs, Hq, Hkv, T, tpb, lens, ids, nb,
                                                 n_items, d, step, o); note_launches(1);
    }
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// Report application (per-block reports buffered on the host, or device lists)
// ---------------------------------------------------------------------------

__global__ void report_apply_kernel(const uint32_t *__restrict__ slots,
                                    const float *__restrict__ psum,
                                    const float *__restrict__ pmax, uint32_t n,
                                    SchedDev d, unsigned long long step)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t s = slots[i] & d.mask;
    if (!d.tact[s]) return;
    d.sum[s] = __fadd_rn(d.sum[s], psum[i]);
    if (pmax[i] > d.mx[s]) d.mx[s] = pmax[i];
    d.last[s] = step;
}

int launch_report_apply(const uint32_t *slots, const float *psum, const float *pmax,
                        uint32_t n, const SchedDev &d, unsigned long long step,
                        cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    report_apply_kernel<<<(n + 255) / 256, 256, 0, s>>>(slots, psum, pmax, n, d, step); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

__global__ void report_batch_kernel(const uint32_t *__restrict__ ids,
                                    const float *__restrict__ w, uint32_t n, SchedDev d,
                                    unsigned long long step, ReportOrder o)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || *o.flag == o.epoch) return;     // aliasing ids: the ordered pass applies them
    record_mass(d, ids[i], w[i], step);
}

int launch_report_batch(const uint32_t *ids, const float *w, uint32_t n,
                        const SchedDev &d, unsigned long long step, const ReportOrder &o,
                        cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    report_batch_kernel<<<(n + 255) / 256, 256, 0, s>>>(ids, w, n, d, step, o); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// Block-mean scores of attention weights [batch][heads][q_len][kv_len] (the
// vLLM hook's reduction), then their reports in (head, block) order
// ---------------------------------------------------------------------------

constexpr int kMeanThreads = 256;
constexpr uint32_t kMeanMaxBlock = 4096;   // tokens per block the kernel accepts

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x)
{
    return __bfloat162float(x);
}

// The mean rounded to the weights' type, as a reduction over a tensor of that
// type returns it.
template <typename T> __device__ __forceinline__ float round_to(float x);
template <> __device__ __forceinline__ float round_to<float>(float x) { return x; }
template <> __device__ __forceinline__ float round_to<__half>(float x)
{
    return __half2float(__float2half_rn(x));
}
template <> __device__ __forceinline__ float round_to<__nv_bfloat16>(float x)
{
    return __bfloat162float(__float2bfloat16_rn(x));
}

constexpr int kMeanRows = 4;          // rows loaded ahead of their sums
constexpr uint32_t kMeanMaxGroups = 8;  // row groups per CTA
// threads that keep all of a B200's 148 SMs streaming (2048 resident each)
constexpr unsigned long long kMeanFillThreads = 148ull * 2048ull;

__device__ __forceinline__ uint4 ld_stream_u4(const void *p)
{
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t vec_word(const uint4 &r, int w)
{
    return w == 0 ? r.x : w == 1 ? r.y : w == 2 ? r.z : r.w;
}

// What one thread loads from one row: V consecutive tokens of type T, as one
// element (V = 1) or one 16-byte vector (V = 16 / sizeof(T)); elem() returns
// token i as fp32 without spilling the vector to local memory.
template <typename T, int V> struct MeanLoad {
    using Raw = uint4;
    static __device__ __forceinline__ Raw load(const T *p) { return ld_stream_u4(p); }
    static __device__ __forceinline__ float elem(const Raw &r, int i);
};
template <typename T> struct MeanLoad<T, 1> {
    using Raw = T;
    static __device__ __forceinline__ Raw load(const T *p) { return *p; }
    static __device__ __forceinline__ float elem(const Raw &r, int) { return to_f32<T>(r); }
};
template <> __device__ __forceinline__ float MeanLoad<float, 4>::elem(const uint4 &r, int i)
{
    return __uint_as_float(vec_word(r, i));
}
template <> __device__ __forceinline__ float MeanLoad<__half, 8>::elem(const uint4 &r, int i)
{
    const uint32_t w = vec_word(r, i >> 1);
    return __half2float(__ushort_as_half((unsigned short)((i & 1) ? w >> 16 : w & 0xFFFFu)));
}
template <> __device__ __forceinline__ float MeanLoad<__nv_bfloat16, 8>::elem(const uint4 &r,
                                                                            int i)
{
    const uint32_t w = vec_word(r, i >> 1);
    return __bfloat162float(
        __ushort_as_bfloat16((unsigned short)((i & 1) ? w >> 16 : w & 0xFFFFu)));
}

// One CTA per (head h, tile of `bpc` consecutive blocks).  The batch x q_len
// rows (batch, then query position) are cut into `rg` row groups of
// ceil(rows / rg) consecutive rows; the CTA's threads form rg groups of
// kMeanThreads / rg, and a thread of group g sums V consecutive tokens
// (coalesced along tokens) over group g's rows in order, kMeanRows loads in
// flight ahead of their sums.  The group sums of each token are then added in
// group order in shared memory, and one thread per block adds its block's
// tokens in order and divides by batch * q_len * block_size: tokens past
// kv_len count as zeros, as in the hook's padded view.  The summation order
// depends on rg and not on V, so the one-element (V = 1) and 16-byte
// (V = 16 / sizeof(T)) instances give bit-identical scores; the 16-byte one
// needs 16-byte-aligned weights and kv_len and block_size multiples of V, so
// every row starts on a 16-byte boundary and a token group lies wholly
// inside or past kv_len.  MINB is the resident CTAs per SM the registers
// are fitted to: 8 for a row-split grid (a short grid gains more from one
// wave than it loses to a few spilled registers), 1 otherwise; it changes no
// arithmetic.
template <typename T, int V, int MINB>
__global__ void __launch_bounds__(kMeanThreads, MINB)
blockmean_kernel(const T *__restrict__ w, uint32_t batch, uint32_t heads, uint32_t q_len,
                 uint32_t kv_len, uint32_t bs, uint32_t nb, uint32_t bpc, uint32_t rg,
                 float denom, float *scores)
{
    using L = MeanLoad<T, V>;
    extern __shared__ float part[];                 // [rg][bpc * bs] token sums per group
    const uint32_t h = blockIdx.y;
    const uint32_t b0 = blockIdx.x * bpc;
    const uint32_t nblk = nb - b0 < bpc ? nb - b0 : bpc;
    const uint32_t t0 = b0 * bs, ntok = nblk * bs, cap = bpc * bs;
    const uint32_t tpg = kMeanThreads / rg;         // threads per row group
    const uint32_t g = threadIdx.x / tpg, c = threadIdx.x % tpg;
    const uint32_t rows = batch * q_len, rpg = (rows + rg - 1) / rg;
    const uint32_t r0 = g * rpg < rows ? g * rpg : rows;
    const uint32_t r1 = r0 + rpg < rows ? r0 + rpg : rows;
    const size_t row_stride = (size_t)q_len * kv_len;            // next query position
    const size_t batch_stride = (size_t)heads * row_stride;      // next batch entry
    const size_t wrap = batch_stride - (size_t)(q_len - 1) * kv_len;
    const T *row0 = w + (size_t)(r0 / q_len) * batch_stride + (size_t)h * row_stride +
                    (size_t)(r0 % q_len) * kv_len;
    for (uint32_t j = c * V; j < ntok; j += tpg * V) {
        const uint32_t t = t0 + j;
        float acc[V];
#pragma unroll
        for (int i = 0; i < V; i++) acc[i] = 0.f;
        if (t < kv_len) {
            // p steps through rows r0 .. r1-1; q is the row's query position
            const T *p = row0 + t;
            uint32_t q = r0 % q_len, r = r0;
            for (; r + kMeanRows <= r1; r += kMeanRows) {
                typename L::Raw v[kMeanRows];
#pragma unroll
                for (int k = 0; k < kMeanRows; k++) {
                    v[k] = L::load(p);
                    p += (++q == q_len) ? (q = 0, wrap) : (size_t)kv_len;
                }
#pragma unroll
                for (int k = 0; k < kMeanRows; k++)
#pragma unroll
                    for (int i = 0; i < V; i++) acc[i] = __fadd_rn(acc[i], L::elem(v[k], i));
            }
            for (; r < r1; r++) {
                const typename L::Raw v = L::load(p);
                p += (++q == q_len) ? (q = 0, wrap) : (size_t)kv_len;
#pragma unroll
                for (int i = 0; i < V; i++) acc[i] = __fadd_rn(acc[i], L::elem(v, i));
            }
        }
#pragma unroll
        for (int i = 0; i < V; i++) part[g * cap + j + i] = acc[i];
    }
    __syncthreads();
    if (rg > 1) {
        for (uint32_t j = threadIdx.x; j < ntok; j += kMeanThreads) {
            float s = part[j];
            for (uint32_t k = 1; k < rg; k++) s = __fadd_rn(s, part[k * cap + j]);
            part[j] = s;
        }
        __syncthreads();
    }
    for (uint32_t k = threadIdx.x; k < nblk; k += kMeanThreads) {
        float s = 0.f;
        for (uint32_t j = 0; j < bs; j++) s = __fadd_rn(s, part[k * bs + j]);
        scores[(size_t)h * nb + b0 + k] = round_to<T>(__fdiv_rn(s, denom));
    }
}

// One warp per block column b; lane l takes head h0 + l of each chunk of 32
// heads, chunks in order.  Lanes whose ids map to one tracker slot (a column
// may give every head the same id) form a group, and the group's lowest lane
// applies the group's reports in head order -- sum, then maximum, then the
// last-hit step, as consecutive tm_notify_attn calls would -- so the results
// round exactly as the sequential calls.  One tracker round trip per slot
// and chunk instead of one per head; __syncwarp orders a chunk's writes
// before the next chunk's reads.  Different columns never share a slot.
__global__ void blockmean_apply_kernel(const float *__restrict__ scores,
                                       const uint32_t *__restrict__ ids, uint32_t heads,
                                       uint32_t nb, SchedDev d, unsigned long long step)
{
    const unsigned long long b =
        ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (b >= nb) return;                              // uniform across the warp
    for (uint32_t h0 = 0; h0 < heads; h0 += 32) {
        const uint32_t h = h0 + lane;
        const uint32_t id = h < heads ? ids[(size_t)h * nb + b] : kNoBlock;
        const float w = h < heads ? scores[(size_t)h * nb + b] : 0.f;
        const bool rec = id != kNoBlock;
        const uint32_t key = rec ? (id & d.mask) : 0xFFFFFFFFu;   // slots are <= mask
        const unsigned grp = __match_any_sync(0xFFFFFFFFu, key);
        const bool lead = rec && lane == __ffs(grp) - 1;
        bool act = false;
        float sum = 0.f, mx = 0.f;
        if (lead) {
            act = d.tact[key];                        // inactive slots ignore reports
            if (act) { sum = d.sum[key]; mx = d.mx[key]; }
        }
        for (int k = 0; k < 32; k++) {                // the group's reports, head order
            const float wk = __shfl_sync(0xFFFFFFFFu, w, k);
            if (act && ((grp >> k) & 1u)) {
                sum = __fadd_rn(sum, wk);
                if (wk > mx) mx = wk;
            }
        }
        if (act) {
            d.sum[key] = sum;
            d.mx[key] = mx;
            d.last[key] = step;
        }
        __syncwarp();
    }
}

int launch_blockmean(const void *w, int dtype, uint32_t batch, uint32_t heads, uint32_t q_len,
                     uint32_t kv_len, uint32_t bs, const uint32_t *ids, float *scores,
                     const SchedDev *d, unsigned long long step, cudaStream_t s)
{
    if (!w || !scores || batch == 0 || heads == 0 || q_len == 0 || kv_len == 0 || bs == 0 ||
        bs > kMeanMaxBlock || dtype < 0 || dtype > 2)
        return ORCHKV_ERR_INVALID;
    const unsigned long long count = (unsigned long long)batch * q_len * bs;
    const float denom = (float)count;         // elements averaged per block
    const uint32_t nb = (kv_len + bs - 1) / bs;
    if (heads > 65535 || count / bs >= (1ull << 29)) return ORCHKV_ERR_INVALID;
    // Row groups from the shape alone (so both kernels sum in one order).
    // Splitting the rows only helps when a thread would otherwise stream
    // more rows than it keeps in flight and the grid is short of the GPU's
    // threads: double the groups while each keeps at least kMeanRows rows,
    // the doubled grid (in 8-token columns) still fits the GPU's resident
    // threads, and the group sums fit 32 KB of shared memory.
    const uint32_t rows = batch * q_len;
    const unsigned long long cols = (unsigned long long)heads * ((kv_len + 7) / 8);
    uint32_t rg = 1;
    while (rg < kMeanMaxGroups && rows >= rg * 2 * kMeanRows &&
           cols * rg * 2 <= kMeanFillThreads && (unsigned long long)rg * 2 * bs <= 8192)
        rg *= 2;
    const uint32_t V = dtype == 2 ? 4 : 8;                      // elements per 16-byte load
    const bool vec = kv_len % V == 0 && bs % V == 0 && ((uintptr_t)w % 16) == 0;
    const uint32_t tile = (kMeanThreads / rg) * (vec ? V : 1);  // tokens per CTA
    const uint32_t bpc = bs >= tile ? 1 : tile / bs;
    const size_t smem = (size_t)rg * bpc * bs * sizeof(float);
    const dim3 grid((nb + bpc - 1) / bpc, heads);
#define OKV_MEAN_LAUNCH(T, VW, MB)                                                         \
    blockmean_kernel<T, VW, MB><<<grid, kMeanThreads, smem, s>>>(                          \
        (const T *)w, batch, heads, q_len, kv_len, bs, nb, bpc, rg, denom, scores)
#define OKV_MEAN_VEC(T, VW)                                                                \
    do {                                                                                   \
        if (rg > 1) OKV_MEAN_LAUNCH(T, VW, 8); else OKV_MEAN_LAUNCH(T, VW, 1);             \
    } while (0)
    if (dtype == 0) {
        if (vec) OKV_MEAN_VEC(__half, 8); else OKV_MEAN_LAUNCH(__half, 1, 1);
    } else if (dtype == 1) {
        if (vec) OKV_MEAN_VEC(__nv_bfloat16, 8); else OKV_MEAN_LAUNCH(__nv_bfloat16, 1, 1);
    } else {
        if (vec) OKV_MEAN_VEC(float, 4); else OKV_MEAN_LAUNCH(float, 1, 1);
    }
#undef OKV_MEAN_VEC
#undef OKV_MEAN_LAUNCH
    note_launches(1);
    if (ids && d) {
        const unsigned long long threads = (unsigned long long)nb * 32;   // a warp per block
        blockmean_apply_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
            scores, ids, heads, nb, *d, step);
        note_launches(1);
    }
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// Token-range mass (the original KVCacheManager's report): block i gets the
// sum over all heads h and tokens t in [start_i, min(end_i, kv_len)) of
// avg[h][t]; blocks whose range is empty are not reported
// ---------------------------------------------------------------------------

// One warp per block: heads in order, lanes strided over the block's tokens
// (coalesced), a warp sum, one tracker record by lane 0.
__global__ void range_mass_kernel(const float *__restrict__ avg, uint32_t heads,
                                  uint32_t kv_len, const uint32_t *__restrict__ start,
                                  const uint32_t *__restrict__ end,
                                  const uint32_t *__restrict__ ids, uint32_t n, SchedDev d,
                                  unsigned long long step, ReportOrder o)
{
    const unsigned lane = threadIdx.x & 31;
    const unsigned long long nw = ((unsigned long long)gridDim.x * blockDim.x) >> 5;
    const bool ordered = *o.flag == o.epoch;
    for (unsigned long long i = ((unsigned long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
         i < n; i += nw) {
        const uint32_t s = start[i];
        const uint32_t e = end[i] < kv_len ? end[i] : kv_len;
        if (s >= e) {                                  // warp-uniform
            if (ordered && lane == 0) o.ids_eff[i] = kNoBlock;
            continue;
        }
        float acc = 0.f;
        if (e - s <= 32) {
            // at most one token per lane: the heads' loads are independent,
            // so the unrolled loop keeps several in flight while the sums
            // stay in head order (the same order as the general loop)
            const uint32_t t = s + lane;
            if (t < e) {
                const float *col = avg + t;
#pragma unroll 8
                for (uint32_t h = 0; h < heads; h++)
                    acc = __fadd_rn(acc, col[(size_t)h * kv_len]);
            }
        } else {
            for (uint32_t h = 0; h < heads; h++) {
                const float *row = avg + (size_t)h * kv_len;
                for (uint32_t t = s + lane; t < e; t += 32) acc = __fadd_rn(acc, row[t]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xFFFFFFFFu, acc, o));
        if (lane == 0) {
            if (ordered) {
                o.ids_eff[i] = ids[i];
                o.mass[i] = acc;
            } else {
                record_mass(d, ids[i], acc, step);
            }
        }
    }
}

int launch_range_mass(const float *avg, uint32_t heads, uint32_t kv_len, const uint32_t *start,
                      const uint32_t *end, const uint32_t *ids, uint32_t n, const SchedDev &d,
                      unsigned long long step, const ReportOrder &o, cudaStream_t s)
{
    if (!avg || !start || !end || !ids || heads == 0 || kv_len == 0) return ORCHKV_ERR_INVALID;
    if (n == 0) return ORCHKV_OK;
    unsigned grid = (unsigned)(((unsigned long long)n * 32 + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    range_mass_kernel<<<grid, 256, 0, s>>>(avg, heads, kv_len, start, end, ids, n, d, step, o);
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// K2: step_done (EMA) and classification sweep
// ---------------------------------------------------------------------------

__device__ __forceinline__ float hotness_of(const SchedDev &d, uint32_t i,
                                            const SchedParams &p,
                                            unsigned long long step)
{
    const unsigned long long last = d.last[i];
    const unsigned long long gap =
        (last == kStepNever) ? step : (step > last ? step - last : 0ull);
    const float rec = gap >= (unsigned long long)kDecayTable ? 0.0f : d.table[gap];
    float freq = 0.0f;
    if (step != 0) {
        freq = __fdiv_rn(__uint2float_rn(d.hits[i]), __ull2float_rn(step));
        if (freq > 1.0f) freq = 1.0f;
    }
    const float t0 = __fmul_rn(p.alpha, d.ema[i]);
    const float t1 = __fmul_rn(p.beta, rec);
    const float t2 = __fmul_rn(p.gamma, freq);
    return __fadd_rn(__fadd_rn(t0, t1), t2);
}

template <bool STEP, bool CLASSIFY>
__global__ void __launch_bounds__(256)
sweep_kernel(SchedDev d, SchedParams p, ClassCounts *counts)
{
    uint32_t n_hot = 0, n_warm = 0, n_cold = 0, n_sink = 0;
    const unsigned long long cstep = STEP ? p.step + 1 : p.step;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < d.cap;
         i += gridDim.x * blockDim.x) {
        const bool ta = d.tact[i] != 0;
        if (STEP && ta) {
            const float e = d.ema[i];
            if (d.last[i] == p.step) {
                d.ema[i] = __fadd_rn(__fmul_rn(p.lambda, e), __fmul_rn(p.one_minus, d.sum[i]));
                d.hits[i] = d.hits[i] + 1;
            } else {
                d.ema[i] = __fmul_rn(e, p.lambda);
            }
            d.sum[i] = 0.0f;
            d.mx[i] = 0.0f;
        }
        if (CLASSIFY) {
            const bool ca = d.cact[i] != 0;
            if (ca && ta) {
                const float h = hotness_of(d, i, p, cstep);
                const uint8_t f = d.cflags[i];
                uint8_t lvl;
                if (f & KV_FLAG_ATTN_SINK) lvl = 0;
                else if (h >= p.th_hot) lvl = 0;
                else if (h >= p.th_warm) lvl = 1;
                else lvl = 2;
                d.hot[i] = h;
                d.heat[i] = lvl;
            }
            if (ca && counts) {
                const uint8_t lvl = d.heat[i];
                n_hot += lvl == 0;
                n_warm += lvl == 1;
                n_cold += lvl == 2;
                n_sink += (d.cflags[i] & KV_FLAG_ATTN_SINK) != 0;
            }
        }
    }
    if (CLASSIFY && counts) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            n_hot += __shfl_xor_sync(0xFFFFFFFFu, n_hot, o);
            n_warm += __shfl_xor_sync(0xFFFFFFFFu, n_warm, o);
            n_cold += __shfl_xor_sync(0xFFFFFFFFu, n_cold, o);
            n_sink += __shfl_xor_sync(0xFFFFFFFFu, n_sink, o);
        }
        if ((threadIdx.x & 31) == 0 && (n_hot | n_warm | n_cold | n_sink)) {
            atomicAdd(&counts->n_hot, n_hot);
            atomicAdd(&counts->n_warm, n_warm);
            atomicAdd(&counts->n_cold, n_cold);
            atomicAdd(&counts->n_sink, n_sink);
        }
    }
}

static unsigned sweep_grid(uint32_t cap)
{
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    unsigned want = (cap + 255) / 256;
    unsigned cap_grid = (unsigned)sms * 8;
    return want < cap_grid ? (want ? want : 1) : cap_grid;
}

int launch_sweep(const SchedDev &d, const SchedParams &p, bool step_done, bool classify,
                 ClassCounts *counts, cudaStream_t s)
{
    if (counts) OKV_CUDA_TRY(cudaMemsetAsync(counts, 0, sizeof(ClassCounts), s));
    const unsigned g = sweep_grid(d.cap);
    if (step_done && classify) sweep_kernel<true, true><<<g, 256, 0, s>>>(d, p, counts);
    else if (step_done) sweep_kernel<true, false><<<g, 256, 0, s>>>(d, p, counts);
    else if (classify) sweep_kernel<false, true><<<g, 256, 0, s>>>(d, p, counts);
    else return ORCHKV_OK;
    note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// Prefetch scan count over the manager's registry
// (src/scheduler/tiered_manager.c:284-312 + prefetch_scheduler.c:131-172)
// ---------------------------------------------------------------------------

__global__ void registry_count_kernel(const uint32_t *__restrict__ reg_slot,
                                      const uint8_t *__restrict__ reg_tier, uint32_t n,
                                      SchedDev d, float th_gpu, float th_dram,
                                      uint32_t *count)
{
    uint32_t c = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += gridDim.x * blockDim.x) {
        const uint8_t t = reg_tier[i];
        if (t == TIER_GPU_HBM || t == TIER_NONE) continue;
        const uint32_t s = reg_slot[i] & d.mask;
        if (!d.tact[s]) continue;
        const float e = d.ema[s];
        if (e >= th_gpu || (e >= th_dram && t != TIER_HOST_DRAM)) c++;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xFFFFFFFFu, c, o);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(count, c);
}

int launch_registry_count(const uint32_t *reg_slot, const uint8_t *reg_tier, uint32_t n,
                          const SchedDev &d, float th_gpu, float th_dram,
                          uint32_t *count, cudaStream_t s)
{
    OKV_CUDA_TRY(cudaMemsetAsync(count, 0, sizeof(uint32_t), s));
    if (n == 0) return ORCHKV_OK;
    unsigned g = (n + 255) / 256;
    if (g > 1184) g = 1184;
    registry_count_kernel<<<g, 256, 0, s>>>(reg_slot, reg_tier, n, d, th_gpu, th_dram, count); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

// ---------------------------------------------------------------------------
// Slot (un)registration: tracker register (attention_tracker.c:179-191),
// classifier register (hotcold_classifier.c:104-116), and resets (:193-202,
// :118-126), applied in list order by one thread (lists are small and may
// repeat a slot).
// ---------------------------------------------------------------------------

__global__ void slot_ops_kernel(const uint32_t *slots, const uint8_t *b, uint32_t n,
                                SchedDev d)
{
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    for (uint32_t j = 0; j < n; j++) {
        const uint32_t s = slots[j] & d.mask;
        const uint8_t op = b[4 * j], fl = b[4 * j + 1], ti = b[4 * j + 2], st = b[4 * j + 3];
        if (op == 0) {
            d.sum[s] = 0.f; d.mx[s] = 0.f; d.ema[s] = 0.f; d.hits[s] = 0;
            d.last[s] = kStepNever; d.tact[s] = 1;
            d.hot[s] = 0.f;
            d.heat[s] = (fl & KV_FLAG_ATTN_SINK) ? 0 : 2;
            d.cflags[s] = fl;
            d.cact[s] = 1;
            d.bflags[s] = fl;
            d.tier[s] = ti;
            d.bstate[s] = st;
        } else if (op == 1) {
            d.sum[s] = 0.f; d.mx[s] = 0.f; d.ema[s] = 0.f; d.hits[s] = 0;
            d.last[s] = 0; d.tact[s] = 0;
            d.hot[s] = 0.f; d.heat[s] = 0; d.cflags[s] = 0; d.cact[s] = 0;
            d.bflags[s] = 0; d.tier[s] = TIER_NONE; d.bstate[s] = 0;
        } else {
            d.tier[s] = ti;
            d.bflags[s] = fl;
            d.bstate[s] = st;
        }
    }
}

int launch_slot_ops(const uint32_t *slots, const uint8_t *b, uint32_t n,
                    const SchedDev &d, cudaStream_t s)
{
    if (n == 0) return ORCHKV_OK;
    slot_ops_kernel<<<1, 32, 0, s>>>(slots, b, n, d); note_launches(1);
    OKV_CUDA_TRY(cudaGetLastError());
    return ORCHKV_OK;
}

}  // namespace okv
