// pybind_module.cpp — the `orchkv_core` Python module.
//
// Same module name, functions, keyword names, defaults, dict keys and error
// behaviour as the reference binding (bindings/orchkv_pybind.cpp:26-416), so
// the reference's Python managers (python/orchkv/kvcache_manager.py,
// python/orchkv/fast_kvcache_manager.py) import it unchanged.  Handles are
// Python ints (uintptr_t), GPU buffers are passed as tensor.data_ptr() ints.
// Everything forwards to liborchkv_b200.so's C ABI.
//
// Additions (not in the reference module): append_token, the tensor-level
// scoring/selection calls and the batched migration calls.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include "orchkv/orchkv_api.h"
#include "orchkv/tiered_manager.h"

namespace py = pybind11;

// Binding-owned block records per manager (bindings/orchkv_pybind.cpp:24).
static std::unordered_map<uintptr_t, std::vector<kv_block_t *>> g_blocks;

template <class T> static T *P(uintptr_t v) { return reinterpret_cast<T *>(v); }

static std::vector<kv_request_ctx_t *> ctx_list(const std::vector<uintptr_t> &v)
{
    std::vector<kv_request_ctx_t *> out(v.size());
    for (size_t i = 0; i < v.size(); i++) out[i] = P<kv_request_ctx_t>(v[i]);
    return out;
}

PYBIND11_MODULE(orchkv_core, m)
{
    m.doc() = "OrchKvCache (B200): tiered KV-cache scheduling and migration on sm_100a";

    py::enum_<StorageTier>(m, "StorageTier")
        .value("GPU_HBM", TIER_GPU_HBM)
        .value("HOST_DRAM", TIER_HOST_DRAM)
        .value("NVM", TIER_NVM)
        .value("SSD", TIER_SSD)
        .value("NONE", TIER_NONE)
        .export_values();

    py::enum_<DataType>(m, "DataType")
        .value("FP16", DTYPE_FP16)
        .value("BF16", DTYPE_BF16)
        .value("FP32", DTYPE_FP32)
        .value("INT8", DTYPE_INT8)
        .value("INT4", DTYPE_INT4)
        .export_values();

    m.attr("OK") = ORCHKV_OK;
    m.attr("ERR_OOM") = ORCHKV_ERR_OOM;
    m.attr("ERR_INVALID") = ORCHKV_ERR_INVALID;
    m.attr("ERR_NOT_FOUND") = ORCHKV_ERR_NOT_FOUND;
    m.attr("ERR_TIER_FULL") = ORCHKV_ERR_TIER_FULL;
    m.attr("ERR_CUDA") = ORCHKV_ERR_CUDA;
    m.attr("ERR_IO") = ORCHKV_ERR_IO;

    py::class_<orchkv_config_t>(m, "Config")
        .def(py::init([]() {
            orchkv_config_t c;
            orchkv_config_default(&c);
            return c;
        }))
        .def_readwrite("gpu_device_id", &orchkv_config_t::gpu_device_id)
        .def_readwrite("gpu_pool_bytes", &orchkv_config_t::gpu_pool_bytes)
        .def_readwrite("dram_pool_bytes", &orchkv_config_t::dram_pool_bytes)
        .def_readwrite("dram_use_pinned", &orchkv_config_t::dram_use_pinned)
        .def_readwrite("num_cuda_streams", &orchkv_config_t::num_cuda_streams)
        .def_readwrite("tokens_per_block", &orchkv_config_t::tokens_per_block)
        .def_readwrite("d_head", &orchkv_config_t::d_head)
        .def_readwrite("dtype", &orchkv_config_t::dtype)
        .def_readwrite("gpu_hwm", &orchkv_config_t::gpu_hwm)
        .def_readwrite("gpu_lwm", &orchkv_config_t::gpu_lwm)
        .def_readwrite("dram_hwm", &orchkv_config_t::dram_hwm)
        .def_readwrite("dram_lwm", &orchkv_config_t::dram_lwm)
        .def_readwrite("orchfs_io_workers", &orchkv_config_t::orchfs_io_workers)
        .def_readwrite("max_blocks_per_head", &orchkv_config_t::max_blocks_per_head)
        .def("__repr__", [](const orchkv_config_t &c) {
            return "<orchkv.Config gpu_pool=" + std::to_string(c.gpu_pool_bytes >> 20) +
                   "MB dram_pool=" + std::to_string(c.dram_pool_bytes >> 20) +
                   "MB d_head=" + std::to_string(c.d_head) + ">";
        });

    m.def("init", &orchkv_init, py::arg("config"), "Initialize the OrchKvCache system");
    m.def("shutdown", &orchkv_shutdown, "Shutdown and free all resources");
    m.def("is_initialized", &orchkv_is_initialized, "Check if the system is initialized");

    m.def("request_create",
          [](uint64_t id, uint32_t L, uint32_t H) -> uintptr_t {
              return reinterpret_cast<uintptr_t>(orchkv_request_create(id, L, H));
          },
          py::arg("request_id"), py::arg("n_layers"), py::arg("n_kv_heads"));
    m.def("request_destroy",
          [](uintptr_t c) { return orchkv_request_destroy(P<kv_request_ctx_t>(c)); },
          py::arg("ctx"));

    m.def("prefill",
          [](uintptr_t c, uint32_t layer, uintptr_t k, uintptr_t v, uint32_t seq) {
              return orchkv_prefill(P<kv_request_ctx_t>(c), layer, P<const void>(k),
                                    P<const void>(v), seq);
          },
          py::arg("ctx"), py::arg("layer"), py::arg("k_ptr"), py::arg("v_ptr"),
          py::arg("seq_len"));
    m.def("get_kv_block",
          [](uintptr_t c, uint32_t l, uint32_t h, uint32_t bi) -> py::tuple {
              void *k = nullptr, *v = nullptr;
              int rc = orchkv_get_kv_block(P<kv_request_ctx_t>(c), l, h, bi, &k, &v);
              return py::make_tuple(rc, reinterpret_cast<uintptr_t>(k),
                                    reinterpret_cast<uintptr_t>(v));
          },
          py::arg("ctx"), py::arg("layer"), py::arg("head"), py::arg("block_idx"));

#define OKV_BLOCK_OP(name, fn)                                                          \
    m.def(name,                                                                         \
          [](uintptr_t c, uint32_t l, uint32_t h, uint32_t bi) {                        \
              return fn(P<kv_request_ctx_t>(c), l, h, bi);                              \
          },                                                                            \
          py::arg("ctx"), py::arg("layer"), py::arg("head"), py::arg("block_idx"))
    OKV_BLOCK_OP("evict_to_dram", orchkv_evict_to_dram);
    OKV_BLOCK_OP("promote_to_gpu", orchkv_promote_to_gpu);
    OKV_BLOCK_OP("evict_to_storage", orchkv_evict_to_storage);
    OKV_BLOCK_OP("promote_from_storage", orchkv_promote_from_storage);
    OKV_BLOCK_OP("evict_cold", orchkv_evict_cold);
#undef OKV_BLOCK_OP
    m.def("storage_flush", &orchkv_storage_flush);

    m.def("get_stats", []() -> py::dict {
        orchkv_stats_t s;
        memset(&s, 0, sizeof(s));
        orchkv_get_stats(&s);
        py::dict d;
        d["gpu_pool_total"] = s.gpu_pool_total;
        d["gpu_pool_used"] = s.gpu_pool_used;
        d["gpu_slabs_total"] = s.gpu_slabs_total;
        d["gpu_slabs_used"] = s.gpu_slabs_used;
        d["dram_pool_total"] = s.dram_pool_total;
        d["dram_pool_used"] = s.dram_pool_used;
        d["dram_slabs_total"] = s.dram_slabs_total;
        d["dram_slabs_used"] = s.dram_slabs_used;
        d["total_blocks"] = s.total_blocks;
        d["blocks_on_gpu"] = s.blocks_on_gpu;
        d["blocks_on_dram"] = s.blocks_on_dram;
        d["blocks_on_nvm"] = s.blocks_on_nvm;
        d["blocks_on_ssd"] = s.blocks_on_ssd;
        d["transfers_d2h"] = s.transfers_d2h;
        d["transfers_h2d"] = s.transfers_h2d;
        d["bytes_d2h"] = s.bytes_d2h;
        d["bytes_h2d"] = s.bytes_h2d;
        d["active_requests"] = s.active_requests;
        return d;
    });

    m.def("tm_create",
          [](uint32_t tracker_cap, float ema_lambda, float alpha, float beta, float gamma,
             uint32_t prefetch_budget, uint32_t schedule_interval_us, float gpu_hwm,
             float gpu_lwm, float dram_hwm, float dram_lwm, uint32_t max_blocks,
             float threshold_to_gpu, float threshold_to_dram, float recency_tau,
             double cooldown_sec, float adjust_step) -> uintptr_t {
              auto *t = new tiered_manager_t();
              tm_config_t cfg;
              tm_config_default(&cfg);
              cfg.tracker_capacity = tracker_cap;
              cfg.ema_lambda = ema_lambda;
              cfg.hcc_params.alpha = alpha;
              cfg.hcc_params.beta = beta;
              cfg.hcc_params.gamma = gamma;
              cfg.hcc_params.recency_tau = recency_tau;
              cfg.prefetch_budget = prefetch_budget;
              cfg.schedule_interval_us = schedule_interval_us;
              cfg.auto_schedule = false;
              cfg.athresh_params.gpu_hwm = gpu_hwm;
              cfg.athresh_params.gpu_lwm = gpu_lwm;
              cfg.athresh_params.dram_hwm = dram_hwm;
              cfg.athresh_params.dram_lwm = dram_lwm;
              cfg.athresh_params.cooldown_sec = cooldown_sec;
              cfg.athresh_params.adjust_step = adjust_step;
              cfg.max_blocks = max_blocks;
              cfg.threshold_to_gpu = threshold_to_gpu;
              cfg.threshold_to_dram = threshold_to_dram;
              int rc = tm_init(t, &cfg);
              if (rc != ORCHKV_OK) {
                  delete t;
                  throw std::runtime_error("tm_init failed: " + std::to_string(rc));
              }
              return reinterpret_cast<uintptr_t>(t);
          },
          py::arg("tracker_cap") = 4096, py::arg("ema_lambda") = 0.9f,
          py::arg("alpha") = 0.5f, py::arg("beta") = 0.3f, py::arg("gamma") = 0.2f,
          py::arg("prefetch_budget") = 16, py::arg("schedule_interval_us") = 1000,
          py::arg("gpu_hwm") = 0.9f, py::arg("gpu_lwm") = 0.7f, py::arg("dram_hwm") = 0.9f,
          py::arg("dram_lwm") = 0.7f, py::arg("max_blocks") = 8192,
          py::arg("threshold_to_gpu") = 0.5f, py::arg("threshold_to_dram") = 0.2f,
          py::arg("recency_tau") = 50.0f, py::arg("cooldown_sec") = 0.5,
          py::arg("adjust_step") = 0.02f);

    m.def("tm_destroy",
          [](uintptr_t tm) {
              auto *t = P<tiered_manager_t>(tm);
              tm_destroy(t);
              auto it = g_blocks.find(tm);
              if (it != g_blocks.end()) {
                  for (auto *b : it->second) delete b;
                  g_blocks.erase(it);
              }
              delete t;
          },
          py::arg("tm"));

    m.def("tm_register_block_id",
          [](uintptr_t tm, uint64_t block_id, int tier, uint8_t flags) -> int {
              auto *b = new kv_block_t();
              std::memset(b, 0, sizeof(*b));
              b->block_id = block_id;
              b->tier = static_cast<StorageTier>(tier);
              b->flags = flags;
              int rc = tm_register_block(P<tiered_manager_t>(tm), b);
              if (rc == ORCHKV_OK) g_blocks[tm].push_back(b);
              else delete b;
              return rc;
          },
          py::arg("tm"), py::arg("block_id"), py::arg("tier") = static_cast<int>(TIER_GPU_HBM),
          py::arg("flags") = 0);

    m.def("tm_set_block_tier",
          [](uintptr_t tm, uint64_t block_id, int tier) {
              tm_set_block_tier_id(P<tiered_manager_t>(tm), block_id, tier);
          },
          py::arg("tm"), py::arg("block_id"), py::arg("tier"));

    m.def("tm_report_attn",
          [](uintptr_t tm, uint64_t id, float w) { tm_notify_attn(P<tiered_manager_t>(tm), id, w); },
          py::arg("tm"), py::arg("block_id"), py::arg("attn_weight"));
    m.def("tm_step_done", [](uintptr_t tm) { tm_step_done(P<tiered_manager_t>(tm)); },
          py::arg("tm"));
    m.def("tm_set_usage",
          [](uintptr_t tm, float g, float d) { tm_set_usage(P<tiered_manager_t>(tm), g, d); },
          py::arg("tm"), py::arg("gpu_ratio"), py::arg("dram_ratio"));
    m.def("tm_schedule_once", [](uintptr_t tm) { tm_schedule_once(P<tiered_manager_t>(tm)); },
          py::arg("tm"));
    m.def("tm_get_block_score",
          [](uintptr_t tm, uint64_t id) -> float { return tm_get_block_score(P<tiered_manager_t>(tm), id); },
          py::arg("tm"), py::arg("block_id"));
    m.def("tm_get_block_heat",
          [](uintptr_t tm, uint64_t id) -> int {
              return static_cast<int>(tm_get_block_heat(P<tiered_manager_t>(tm), id));
          },
          py::arg("tm"), py::arg("block_id"));
    m.def("tm_start", [](uintptr_t tm) { return tm_start(P<tiered_manager_t>(tm)); }, py::arg("tm"));
    m.def("tm_stop", [](uintptr_t tm) { tm_stop(P<tiered_manager_t>(tm)); }, py::arg("tm"));
    m.def("tm_set_policy",
          [](uintptr_t tm, float a, float b, float g) { tm_set_policy(P<tiered_manager_t>(tm), a, b, g); },
          py::arg("tm"), py::arg("alpha"), py::arg("beta"), py::arg("gamma"));

    m.def("tm_get_stats",
          [](uintptr_t tm) -> py::dict {
              auto *t = P<tiered_manager_t>(tm);
              tm_stats_t s;
              tm_get_stats(t, &s);
              float th_hot = 0.f, th_warm = 0.f;
              uint64_t up = 0, down = 0;
              tm_get_threshold_state(t, &th_hot, &th_warm, &up, &down);
              py::dict d;
              d["schedule_cycles"] = s.schedule_cycles;
              d["gpu_demotes"] = s.gpu_demotes;
              d["dram_demotes"] = s.dram_demotes;
              d["prefetches_dispatched"] = s.prefetches_dispatched;
              d["gpu_used_ratio"] = s.gpu_used_ratio;
              d["dram_used_ratio"] = s.dram_used_ratio;
              d["blocks_migrated"] = s.migration_stats.blocks_migrated;
              d["migration_errors"] = s.migration_stats.op_errors;
              d["prefetch_hits"] = s.prefetch_stats.prefetch_hits;
              d["prefetch_wasted"] = s.prefetch_stats.prefetch_wasted;
              d["prefetch_hit_rate"] = s.prefetch_stats.hit_rate;
              d["n_hot"] = s.hcc_stats.n_hot;
              d["n_warm"] = s.hcc_stats.n_warm;
              d["n_cold"] = s.hcc_stats.n_cold;
              d["threshold_adj_up"] = up;
              d["threshold_adj_down"] = down;
              d["threshold_hot"] = th_hot;
              d["threshold_warm"] = th_warm;
              return d;
          },
          py::arg("tm"));

    // ---- additions -----------------------------------------------------------
    m.def("append_token",
          [](uintptr_t c, uint32_t layer, uintptr_t k, uintptr_t v) {
              return orchkv_append_token(P<kv_request_ctx_t>(c), layer, P<const void>(k),
                                         P<const void>(v));
          },
          py::arg("ctx"), py::arg("layer"), py::arg("k_ptr"), py::arg("v_ptr"));
    m.def("append_token_batch",
          [](const std::vector<uintptr_t> &ctxs, uintptr_t k, uintptr_t v) {
              auto l = ctx_list(ctxs);
              return orchkv_append_token_batch(l.data(), (uint32_t)l.size(), P<const void>(k),
                                               P<const void>(v));
          },
          py::arg("ctxs"), py::arg("k_ptr"), py::arg("v_ptr"));
    m.def("block_checksums",
          [](uintptr_t ids, uint32_t n, uintptr_t out, uintptr_t tiers) {
              return orchkv_block_checksums(P<const uint32_t>(ids), n,
                                            P<unsigned long long>(out), P<uint8_t>(tiers));
          },
          py::arg("block_ids_ptr"), py::arg("n"), py::arg("out_ptr"), py::arg("tiers_ptr") = 0);
    m.def("block_id_table",
          [](const std::vector<uintptr_t> &ctxs, uint32_t row_len, uintptr_t out) {
              auto l = ctx_list(ctxs);
              return orchkv_block_id_table(l.data(), (uint32_t)l.size(), row_len, P<uint32_t>(out));
          },
          py::arg("ctxs"), py::arg("row_len"), py::arg("out_ptr"));
    m.def("evict_batch_to_dram",
          [](uintptr_t ids, uintptr_t count, uint32_t max_n, uintptr_t result) {
              return orchkv_evict_batch_to_dram(P<const uint32_t>(ids), P<const uint32_t>(count),
                                                max_n, P<uint32_t>(result));
          },
          py::arg("ids_ptr"), py::arg("count_ptr"), py::arg("max_n"), py::arg("result_ptr") = 0);
    m.def("promote_batch_to_gpu",
          [](uintptr_t ids, uintptr_t count, uint32_t max_n, uintptr_t result) {
              return orchkv_promote_batch_to_gpu(P<const uint32_t>(ids), P<const uint32_t>(count),
                                                 max_n, P<uint32_t>(result));
          },
          py::arg("ids_ptr"), py::arg("count_ptr"), py::arg("max_n"), py::arg("result_ptr") = 0);
#define OKV_STORAGE_BATCH(name, fn)                                                     \
    m.def(name,                                                                         \
          [](uintptr_t c, const std::vector<uint32_t> &lhb) -> py::tuple {              \
              uint32_t res[2] = {0, 0};                                                 \
              const uint32_t n = (uint32_t)(lhb.size() / 3);                            \
              int rc = fn(P<kv_request_ctx_t>(c), lhb.data(), n, res);                  \
              return py::make_tuple(rc, res[0], res[1]);                                \
          },                                                                            \
          py::arg("ctx"), py::arg("lhb"))
    OKV_STORAGE_BATCH("evict_batch_to_storage", orchkv_evict_batch_to_storage);
    OKV_STORAGE_BATCH("promote_batch_from_storage", orchkv_promote_batch_from_storage);
    OKV_STORAGE_BATCH("evict_cold_batch", orchkv_evict_cold_batch);
#undef OKV_STORAGE_BATCH
    m.def("swap_batch",
          [](uintptr_t evict_ids, uintptr_t evict_count, uint32_t max_evict, uintptr_t promote_ids,
             uintptr_t promote_count, uint32_t max_promote, uintptr_t result) {
              return orchkv_swap_batch(P<const uint32_t>(evict_ids), P<const uint32_t>(evict_count),
                                       max_evict, P<const uint32_t>(promote_ids),
                                       P<const uint32_t>(promote_count), max_promote,
                                       P<uint32_t>(result));
          },
          py::arg("evict_ids_ptr"), py::arg("evict_count_ptr"), py::arg("max_evict"),
          py::arg("promote_ids_ptr"), py::arg("promote_count_ptr"), py::arg("max_promote"),
          py::arg("result_ptr") = 0);
    m.def("attach_scheduler",
          [](uintptr_t tm) { return orchkv_attach_scheduler(P<tiered_manager_t>(tm)); },
          py::arg("tm"));
    m.def("set_stream", [](uintptr_t s) { return orchkv_set_stream(P<void>(s)); }, py::arg("stream"));
    m.def("sync", &orchkv_sync);
    m.def("tm_set_stream",
          [](uintptr_t tm, uintptr_t s) { return tm_set_stream(P<tiered_manager_t>(tm), P<void>(s)); },
          py::arg("tm"), py::arg("stream"));
    m.def("tm_sync", [](uintptr_t tm) { return tm_sync(P<tiered_manager_t>(tm)); }, py::arg("tm"));
    m.def("tm_capacity", [](uintptr_t tm) { return tm_capacity(P<tiered_manager_t>(tm)); },
          py::arg("tm"));
    m.def("tm_report_attn_probs",
          [](uintptr_t tm, uintptr_t probs, uint32_t n_rows, uint32_t hq, uint32_t hkv,
             uint32_t row_len, uint32_t tpb, uintptr_t ids, uintptr_t lens) {
              return tm_report_attn_probs(P<tiered_manager_t>(tm), P<const float>(probs), n_rows,
                                          hq, hkv, row_len, tpb, P<const uint32_t>(lens),
                                          P<const uint32_t>(ids));
          },
          py::arg("tm"), py::arg("probs_ptr"), py::arg("n_rows"), py::arg("n_q_heads"),
          py::arg("n_kv_heads"), py::arg("row_len"), py::arg("tokens_per_block"),
          py::arg("block_ids_ptr"), py::arg("lens_ptr") = 0);
    m.def("tm_report_attn_ranges",
          [](uintptr_t tm, uintptr_t avg, uint32_t heads, uint32_t kv_len, uintptr_t starts,
             uintptr_t ends, uintptr_t ids, uint32_t n) {
              return tm_report_attn_ranges(P<tiered_manager_t>(tm), P<const float>(avg), heads,
                                           kv_len, P<const uint32_t>(starts),
                                           P<const uint32_t>(ends), P<const uint32_t>(ids), n);
          },
          py::arg("tm"), py::arg("avg_ptr"), py::arg("heads"), py::arg("kv_len"),
          py::arg("starts_ptr"), py::arg("ends_ptr"), py::arg("block_ids_ptr"), py::arg("n"));
    m.def("tm_report_attn_batch_dev",
          [](uintptr_t tm, uintptr_t ids, uintptr_t weights, uint32_t n) {
              return tm_report_attn_batch_dev(P<tiered_manager_t>(tm), P<const uint32_t>(ids),
                                              P<const float>(weights), n);
          },
          py::arg("tm"), py::arg("block_ids_ptr"), py::arg("weights_ptr"), py::arg("n"));
    m.def("tm_stage_input_async",
          [](uintptr_t tm, uintptr_t host, size_t bytes) {
              return tm_stage_input_async(P<tiered_manager_t>(tm), P<const void>(host), bytes);
          },
          py::arg("tm"), py::arg("host_ptr"), py::arg("nbytes"));
    m.def("tm_report_attn_blockmean",
          [](uintptr_t tm, uintptr_t weights, int dtype, uint32_t batch, uint32_t heads,
             uint32_t q_len, uint32_t kv_len, uint32_t block_size, uintptr_t ids,
             uintptr_t scores) {
              return tm_report_attn_blockmean(P<tiered_manager_t>(tm), P<const void>(weights),
                                              dtype, batch, heads, q_len, kv_len, block_size,
                                              P<const uint32_t>(ids), P<float>(scores));
          },
          py::arg("tm"), py::arg("weights_ptr"), py::arg("dtype"), py::arg("batch"),
          py::arg("heads"), py::arg("q_len"), py::arg("kv_len"), py::arg("block_size"),
          py::arg("block_ids_ptr"), py::arg("scores_ptr"));
    m.def("tm_step_and_classify",
          [](uintptr_t tm) { return tm_step_and_classify(P<tiered_manager_t>(tm)); }, py::arg("tm"));
    m.def("tm_select_victims",
          [](uintptr_t tm, uint32_t k, uintptr_t out, uintptr_t count) {
              return tm_select_victims(P<tiered_manager_t>(tm), k, P<uint32_t>(out), P<uint32_t>(count));
          },
          py::arg("tm"), py::arg("k"), py::arg("out_ptr"), py::arg("count_ptr"));
    m.def("tm_select_victims_masked",
          [](uintptr_t tm, uint32_t k, uintptr_t eligible, uintptr_t out, uintptr_t count) {
              return tm_select_victims_masked(P<tiered_manager_t>(tm), k,
                                              P<const uint8_t>(eligible), P<uint32_t>(out),
                                              P<uint32_t>(count));
          },
          py::arg("tm"), py::arg("k"), py::arg("eligible_ptr"), py::arg("out_ptr"),
          py::arg("count_ptr"));
    m.def("copy_token_blocks",
          [](const std::vector<uintptr_t> &bufs, uint32_t n_heads, uint64_t head_stride,
             uint32_t row_bytes, uint32_t block_tokens, uint32_t n_tokens, uintptr_t blocks,
             uint32_t n_blocks, uintptr_t store, int dir, uintptr_t stream, uintptr_t slots) {
              std::vector<void *> b(bufs.size());
              for (size_t i = 0; i < bufs.size(); i++) b[i] = reinterpret_cast<void *>(bufs[i]);
              return orchkv_copy_token_blocks(b.data(), (uint32_t)b.size(), n_heads, head_stride,
                                              row_bytes, block_tokens, n_tokens,
                                              P<const uint32_t>(blocks), n_blocks, P<void>(store),
                                              P<const uint32_t>(slots), dir, P<void>(stream));
          },
          py::arg("bufs"), py::arg("n_heads"), py::arg("head_stride_bytes"), py::arg("row_bytes"),
          py::arg("block_tokens"), py::arg("n_tokens"), py::arg("blocks_ptr"),
          py::arg("n_blocks"), py::arg("store_ptr"), py::arg("dir"), py::arg("stream") = 0,
          py::arg("slots_ptr") = 0);
    m.def("tm_select_prefetch",
          [](uintptr_t tm, uint32_t k, float thg, float thd, uintptr_t out, uintptr_t count) {
              return tm_select_prefetch(P<tiered_manager_t>(tm), k, thg, thd, P<uint32_t>(out),
                                        P<uint32_t>(count));
          },
          py::arg("tm"), py::arg("k"), py::arg("threshold_to_gpu"), py::arg("threshold_to_dram"),
          py::arg("out_ptr"), py::arg("count_ptr"));
}
