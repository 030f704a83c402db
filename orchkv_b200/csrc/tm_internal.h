// tm_internal.h — host object behind tiered_manager_t.impl.
#pragma once

#include <pthread.h>

#include <atomic>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "kernels.h"
#include "orchkv/tiered_manager.h"

struct PendingReport {
    float sum = 0.0f;
    float max = 0.0f;
};

struct RegShadow {
    uint8_t tier, flags, state;
};

struct RegEntry {
    uint32_t slot;
    uint8_t tier;
};

// A host input uploaded ahead of the report call that consumes it
// (tm_stage_input_async).
struct StagedInput {
    const void *host = nullptr;
    size_t bytes = 0;
    char *dev = nullptr;
    size_t cap = 0;
    cudaEvent_t ready = nullptr;      // the upload finished (on the staging stream)
    cudaEvent_t consumed = nullptr;   // the consuming report's kernels finished
    bool pending = false;             // uploaded (or uploading), not yet consumed
    bool in_use = false;              // taken by the report call being launched
    unsigned long long seq = 0;
};

// Ranks a selection can split ties over: the tie all-gather lands in the 48
// words of `small` after its first 16.
constexpr int kMaxSelectRanks = 48;

struct TmImpl {
    std::mutex mu;
    int device = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;

    // tracker / classifier parameters
    uint32_t cap = 0, mask = 0;
    float lambda = 0.9f;
    unsigned long long step = 0;
    float alpha = 0.5f, beta = 0.3f, gamma = 0.2f, tau = 50.0f;
    float table[512];

    // threshold controller (adaptive_threshold.h:31-58)
    float th_hot = 0.5f, th_warm = 0.2f;
    float min_hot = 0.2f, max_hot = 0.9f, min_warm = 0.05f, max_warm = 0.5f;
    float gpu_hwm = 0.9f, gpu_lwm = 0.7f, dram_hwm = 0.9f, dram_lwm = 0.7f;
    float adjust_step = 0.02f;
    double cooldown_sec = 0.5, last_adjust = 0.0;
    uint64_t adj_up = 0, adj_down = 0, demote_checks = 0;
    float gpu_ratio = 0.0f, dram_ratio = 0.0f;

    // eviction policy (eviction_policy.h:40-56)
    float w_heat = 0.7f, w_lru = 0.3f;
    kv_block_t *lru_head = nullptr, *lru_tail = nullptr;
    uint32_t lru_count = 0;

    // prefetch scheduler counters (prefetch_scheduler.h:58-84)
    uint32_t prefetch_budget = 16;
    float th_gpu_pf = 0.5f, th_dram_pf = 0.2f;
    uint32_t heap_size = 0, tracked = 0;
    uint64_t total_scanned = 0, total_enqueued = 0, total_dispatched = 0;
    uint64_t prefetch_hits = 0, prefetch_wasted = 0;

    // migration engine (migration_engine.h:76-89)
    mig_transfer_fn transfer_fn = nullptr;
    void *transfer_ctx = nullptr;
    uint64_t op_count[MIGRATE_OP_COUNT] = {0}, op_bytes[MIGRATE_OP_COUNT] = {0};
    uint64_t mig_errors = 0, blocks_migrated = 0;

    // manager (tiered_manager.h:101-144)
    tm_alloc_fn alloc_fn = nullptr;
    tm_free_fn free_fn = nullptr;
    void *alloc_ctx = nullptr;
    size_t block_data_size = 0;
    uint32_t schedule_interval_us = 1000, demote_batch_size = 8, prefetch_batch_size = 8;
    uint32_t max_blocks = 4096;
    std::vector<kv_block_t *> blocks;
    std::vector<RegShadow> shadow;
    uint64_t schedule_cycles = 0, gpu_demotes = 0, dram_demotes = 0, prefetches_dispatched = 0;
    std::atomic<bool> running{false};
    pthread_t thread;

    // device state
    char *dev_block = nullptr;
    okv::SchedDev d;
    okv::SelectScratch sc;
    okv::ClassCounts *counts = nullptr;
    uint32_t *small = nullptr;    // device scratch words
    uint32_t *h_small = nullptr;  // pinned

    // pinned host mirrors for getters
    float *m_hot = nullptr;
    uint8_t *m_heat = nullptr, *m_cact = nullptr, *m_cflags = nullptr;
    bool mirror_dirty = true;

    // pending host-side work
    std::vector<uint32_t> ops_slot;
    std::vector<uint8_t> ops_b;
    std::unordered_map<uint32_t, PendingReport> pending;
    char *up_host = nullptr, *up_dev = nullptr;
    size_t up_cap = 0;
    std::vector<RegEntry> reg_tmp;
    char *reg_host = nullptr, *reg_dev = nullptr;
    size_t reg_cap = 0;
    char *in_stage = nullptr;     // device copies of host inputs to tm_report_attn_probs
    size_t in_stage_cap = 0;
    // ordering of tensor-level reports whose ids share slots (okv::ReportOrder)
    uint32_t *report_mark = nullptr;   // [cap], inside dev_block
    uint32_t *report_flag = nullptr;   // one word, inside dev_block
    uint32_t report_epoch = 0;
    char *report_scratch = nullptr;    // per-entry ids and masses of an ordered call
    size_t report_scratch_cap = 0;
    // opt-in device timing of tm_report_attn_probs' launches (tm_profile_reports):
    // before the duplicate-slot pass, before the score kernel, after it, after
    // the ordered pass
    bool rep_prof = false;
    cudaEvent_t rep_ev[4] = {};
    // inputs staged ahead of their report (two slots, consumed oldest first)
    StagedInput early[2];
    cudaStream_t early_copy = nullptr;
    unsigned long long early_seq = 0;

    // multi-GPU selection hooks (set by the comm layer)
    okv::hist_reduce_fn comm_reduce = nullptr;
    okv::tie_gather_fn comm_gather = nullptr;
    void *comm_ctx = nullptr;
    int comm_rank = 0, comm_world = 1;      // comm_world <= kMaxSelectRanks
};

TmImpl *tm_impl(const tiered_manager_t *m);
// data plane hook (api.cu): detach m if it is the attached manager
extern "C" __attribute__((visibility("hidden"))) void okv_manager_destroyed(tiered_manager_t *m);
// data plane hook (api.cu): ORCHKV_ERR_CUDA when a checked build met an
// out-of-range index
extern "C" __attribute__((visibility("hidden"))) int okv_data_plane_check(void);
int tm_flush_locked(TmImpl *t);
int tm_refresh_mirror_locked(TmImpl *t);
