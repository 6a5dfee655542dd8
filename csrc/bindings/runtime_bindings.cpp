// pybind11 surface of bloom_b200._runtime (host C++ runtime; no CUDA needed).
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "../runtime/block_manager.h"
#include "../runtime/scheduler.h"

namespace py = pybind11;
using namespace bloom::rt;

namespace {

template <typename T>
T* host_ptr(const torch::Tensor& t, at::ScalarType st, const char* name) {
  TORCH_CHECK(t.device().is_cpu(), name, " must be a host tensor");
  TORCH_CHECK(t.scalar_type() == st, name, " has the wrong dtype");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  return reinterpret_cast<T*>(t.data_ptr());
}

py::dict metrics_dict(const PoolMetrics& m) {
  py::dict d;
  d["total_blocks"] = m.total_blocks;
  d["free_blocks"] = m.free_blocks;
  d["active_blocks"] = m.active_blocks;
  d["cached_blocks"] = m.cached_blocks;
  d["hits"] = m.hits;
  d["misses"] = m.misses;
  d["evictions"] = m.evictions;
  d["reuses"] = m.reuses;
  return d;
}

}  // namespace

void register_cpu_ops(py::module_& m);  // csrc/runtime/cpu_ops.cpp
void register_gguf(py::module_& m);     // csrc/runtime/gguf.cpp
void register_json(py::module_& m);     // csrc/runtime/json_dfa.cpp
void register_plugin(py::module_& m);   // csrc/runtime/plugin_loader.cpp
void register_quantize(py::module_& m); // csrc/runtime/quantize.cpp
void register_admission(py::module_& m); // csrc/runtime/admission.cpp
void register_schema(py::module_& m);    // csrc/runtime/schema_matcher.cpp
void register_model_store(py::module_& m);  // csrc/runtime/model_store.cpp
void register_image(py::module_& m);        // csrc/runtime/model_store.cpp (PNG scanlines)
void register_media_encode(py::module_& m); // csrc/runtime/media_encode.cpp (GIF / PNG output)

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "bloom_b200 host runtime: KV block manager, in-flight batching scheduler, CPU kernels";

  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int, int, bool>(), py::arg("num_blocks"), py::arg("block_size") = 16,
           py::arg("enable_prefix_caching") = true)
      .def_property_readonly("num_available", &BlockManager::num_available)
      .def_property_readonly("block_size", &BlockManager::block_size)
      .def("match_prefix",
           [](BlockManager& bm, const std::vector<int32_t>& tokens, int max_tokens) {
             std::vector<int32_t> table;
             std::vector<uint64_t> hashes;
             const int n = bm.match_prefix(tokens, max_tokens, table, hashes);
             return py::make_tuple(n, table, hashes);
           })
      .def("allocate",
           [](BlockManager& bm, std::vector<int32_t> table, int num_tokens) {
             const bool ok = bm.ensure_capacity(table, num_tokens);
             return py::make_tuple(ok, table);
           })
      .def("commit",
           [](BlockManager& bm, const std::vector<int32_t>& tokens, int num_computed, const std::vector<int32_t>& table,
              std::vector<uint64_t> hashes) {
             bm.commit_full_blocks(tokens, num_computed, table, hashes);
             return hashes;
           })
      .def("release",
           [](BlockManager& bm, std::vector<int32_t> table, std::vector<uint64_t> hashes) {
             bm.release(table, hashes);
           })
      .def("truncate",
           [](BlockManager& bm, std::vector<int32_t> table, std::vector<uint64_t> hashes, int num_tokens) {
             bm.truncate(table, hashes, num_tokens);
             return py::make_tuple(table, hashes);
           })
      .def("evict_cached", &BlockManager::evict_cached)
      .def("reset_prefix_cache", &BlockManager::reset_prefix_cache)
      .def("refcount", &BlockManager::refcount)
      .def("metrics", [](const BlockManager& bm) { return metrics_dict(bm.metrics()); });

  py::class_<SamplingParams>(m, "SamplingParams")
      .def(py::init<>())
      .def_readwrite("temperature", &SamplingParams::temperature)
      .def_readwrite("top_p", &SamplingParams::top_p)
      .def_readwrite("top_k", &SamplingParams::top_k)
      .def_readwrite("seed", &SamplingParams::seed)
      .def_readwrite("max_tokens", &SamplingParams::max_tokens)
      .def_readwrite("min_tokens", &SamplingParams::min_tokens)
      .def_readwrite("ignore_eos", &SamplingParams::ignore_eos)
      .def_readwrite("stop_token_ids", &SamplingParams::stop_token_ids);

  py::class_<SchedulerConfig>(m, "SchedulerConfig")
      .def(py::init<>())
      .def_readwrite("max_num_seqs", &SchedulerConfig::max_num_seqs)
      .def_readwrite("max_num_batched_tokens", &SchedulerConfig::max_num_batched_tokens)
      .def_readwrite("max_model_len", &SchedulerConfig::max_model_len)
      .def_readwrite("chunked_prefill", &SchedulerConfig::chunked_prefill)
      .def_readwrite("eos_token_ids", &SchedulerConfig::eos_token_ids)
      .def_readwrite("spec_len", &SchedulerConfig::spec_len)
      .def_readwrite("victim_policy", &SchedulerConfig::victim_policy)
      .def_readwrite("max_preemptions_per_request", &SchedulerConfig::max_preemptions_per_request)
      .def_readwrite("priority_preempt_ms", &SchedulerConfig::priority_preempt_ms)
      .def_readwrite("kv_admission_threshold", &SchedulerConfig::kv_admission_threshold)
      .def_readwrite("swap_slots", &SchedulerConfig::swap_slots)
      .def_readwrite("lc_policy", &SchedulerConfig::lc_policy)
      .def_readwrite("lc_window_tokens", &SchedulerConfig::lc_window_tokens)
      .def_readwrite("lc_max_context", &SchedulerConfig::lc_max_context)
      .def_readwrite("lc_shift", &SchedulerConfig::lc_shift)
      .def_readwrite("lc_target_free", &SchedulerConfig::lc_target_free);

  py::class_<StepMeta>(m, "StepMeta")
      .def_readonly("num_tokens", &StepMeta::num_tokens)
      .def_readonly("num_decode", &StepMeta::num_decode)
      .def_readonly("decode_q_len", &StepMeta::decode_q_len)
      .def_readonly("num_real_decode", &StepMeta::num_real_decode)
      .def_readonly("num_prefill", &StepMeta::num_prefill)
      .def_readonly("num_tiles", &StepMeta::num_tiles)
      .def_readonly("num_logits", &StepMeta::num_logits)
      .def_readonly("num_real_logits", &StepMeta::num_real_logits)
      .def_readonly("max_decode_blocks", &StepMeta::max_decode_blocks)
      .def_readonly("num_preempted", &StepMeta::num_preempted)
      .def_readonly("all_greedy", &StepMeta::all_greedy)
      .def_readonly("off_input_ids", &StepMeta::off_input_ids)
      .def_readonly("off_slot_mapping", &StepMeta::off_slot_mapping)
      .def_readonly("off_positions", &StepMeta::off_positions)
      .def_readonly("off_decode_seq_lens", &StepMeta::off_decode_seq_lens)
      .def_readonly("off_decode_block_table", &StepMeta::off_decode_block_table)
      .def_readonly("off_prefill_ctx_lens", &StepMeta::off_prefill_ctx_lens)
      .def_readonly("off_prefill_cu_q", &StepMeta::off_prefill_cu_q)
      .def_readonly("off_prefill_block_table", &StepMeta::off_prefill_block_table)
      .def_readonly("off_tile_seq", &StepMeta::off_tile_seq)
      .def_readonly("off_tile_start", &StepMeta::off_tile_start)
      .def_readonly("off_logits_rows", &StepMeta::off_logits_rows)
      .def_readonly("off_top_k", &StepMeta::off_top_k)
      .def_readonly("off_temperature", &StepMeta::off_temperature)
      .def_readonly("off_top_p", &StepMeta::off_top_p)
      .def_readonly("off_draft_ids", &StepMeta::off_draft_ids)
      .def_readonly("off_seeds", &StepMeta::off_seeds)
      .def_readonly("off_offsets", &StepMeta::off_offsets)
      .def_readonly("used_words", &StepMeta::used_words);

  m.def("arena_layout", &arena_layout, py::arg("T"), py::arg("Bd"), py::arg("Sp"), py::arg("NT"), py::arg("NL"),
        py::arg("MB"), py::arg("q_len") = 1);
  m.def("ngram_propose", &ngram_propose, py::arg("tokens"), py::arg("k"), py::arg("max_order") = 4,
        py::arg("min_order") = 1);

  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init<const SchedulerConfig&, int, int, bool>(), py::arg("config"), py::arg("num_blocks"),
           py::arg("block_size") = 16, py::arg("enable_prefix_caching") = true)
      .def(
          "set_arena",
          [](Scheduler& s, const torch::Tensor& arena, int max_tokens, int max_seqs, int max_blocks) {
            Arena a;
            a.base = host_ptr<int32_t>(arena, at::kInt, "arena");
            a.capacity = arena.numel();
            a.max_tokens = max_tokens;
            a.max_seqs = max_seqs;
            a.max_blocks = max_blocks;
            const StepMeta worst = arena_layout(max_tokens, max_seqs, max_seqs, max_tokens / 64 + max_seqs,
                                                max_tokens + max_seqs, max_blocks);
            TORCH_CHECK(worst.used_words <= a.capacity, "arena too small: need ", worst.used_words, " words");
            s.set_arena(a);
          },
          py::keep_alive<1, 2>())
      .def("set_decode_buckets", &Scheduler::set_decode_buckets)
      .def("add_request", &Scheduler::add_request, py::arg("prompt"), py::arg("params"), py::arg("priority") = 0)
      .def("abort", &Scheduler::abort)
      .def("maintain_long_context", &Scheduler::maintain_long_context)
      .def("visible_blocks", &Scheduler::visible_blocks)
      .def("has_unfinished", &Scheduler::has_unfinished)
      .def_property_readonly("num_waiting", &Scheduler::num_waiting)
      .def_property_readonly("num_running", &Scheduler::num_running)
      .def_property_readonly("total_preemptions", &Scheduler::total_preemptions)
      .def_property_readonly("admissions_deferred", &Scheduler::admissions_deferred)
      .def_property_readonly("priority_preemptions", &Scheduler::priority_preemptions)
      .def("set_clock_ms", &Scheduler::set_clock_ms)
      .def("take_swap_ins", &Scheduler::take_swap_ins)
      .def("take_swap_outs", &Scheduler::take_swap_outs)
      .def_property_readonly("free_swap_slots", &Scheduler::free_swap_slots)
      .def_property_readonly("total_swap_outs", &Scheduler::total_swap_outs)
      .def("export_sequence",
           [](const Scheduler& s, int64_t id) {
             const Scheduler::SeqState st = s.export_sequence(id);
             py::dict d;
             d["tokens"] = st.tokens;
             d["num_prompt"] = st.num_prompt;
             d["num_computed"] = st.num_computed;
             d["blocks"] = st.blocks;
             d["priority"] = st.priority;
             d["params"] = st.sp;
             return d;
           })
      .def("import_sequence", &Scheduler::import_sequence, py::arg("tokens"), py::arg("num_prompt"),
           py::arg("num_computed"), py::arg("params"), py::arg("priority") = 0)
      .def("now_ms", &Scheduler::now_ms)
      .def("kv_utilization", &Scheduler::kv_utilization)
      .def("num_preemptions",
           [](const Scheduler& s, int64_t id) {
             const Sequence* q = s.find(id);
             return q == nullptr ? -1 : q->num_preemptions;
           })
      .def("schedule", &Scheduler::schedule, py::call_guard<py::gil_scoped_release>())
      .def("update",
           [](Scheduler& s, const torch::Tensor& sampled, int n) {
             const int32_t* p = host_ptr<int32_t>(sampled, at::kInt, "sampled");
             TORCH_CHECK(sampled.numel() >= n, "sampled smaller than n");
             std::vector<Event> ev;
             {
               py::gil_scoped_release nogil;
               ev = s.update(p, n);
             }
             py::list out;
             for (const Event& e : ev) out.append(py::make_tuple(e.seq_id, e.token, e.finished, e.finish_reason));
             return out;
           })
      .def("sequence_tokens",
           [](const Scheduler& s, int64_t id) {
             const Sequence* q = s.find(id);
             if (q == nullptr) return std::vector<int32_t>();
             return q->tokens;
           })
      .def("num_cached_prefix",
           [](const Scheduler& s, int64_t id) {
             const Sequence* q = s.find(id);
             return q == nullptr ? 0 : q->num_cached_prefix;
           })
      .def("sampling_ids", &Scheduler::sampling_ids)
      .def("fail_scheduled", &Scheduler::fail_scheduled)
      .def(
          "enable_cachemesh",
          [](Scheduler& s, const torch::Tensor& l2, int64_t block_bytes, const std::string& l3_dir,
             int64_t l3_max_blocks, const std::string& ns) {
            TORCH_CHECK(l2.device().is_cpu() && l2.scalar_type() == at::kByte && l2.is_contiguous(),
                        "cachemesh: L2 must be a contiguous uint8 host tensor (pinned)");
            TORCH_CHECK(block_bytes > 0 && l2.numel() % block_bytes == 0, "cachemesh: L2 size not a block multiple");
            CacheMeshConfig c;
            c.l2_slots = l2.numel() / block_bytes;
            c.block_bytes = block_bytes;
            c.l3_dir = l3_dir;
            c.l3_max_blocks = l3_max_blocks;
            c.name_space = ns;
            s.enable_cachemesh(c, l2.data_ptr<uint8_t>());
          },
          py::arg("l2"), py::arg("block_bytes"), py::arg("l3_dir") = "", py::arg("l3_max_blocks") = 0,
          py::arg("namespace") = "default", py::keep_alive<1, 2>())
      .def("take_offloads",
           [](Scheduler& s) {
             std::vector<std::pair<int, int>> v;
             for (auto& c : s.blocks().take_offloads()) v.emplace_back(c.block, c.slot);
             return v;
           })
      .def("take_restores",
           [](Scheduler& s) {
             std::vector<std::pair<int, int>> v;
             for (auto& c : s.blocks().take_restores()) v.emplace_back(c.block, c.slot);
             return v;
           })
      .def("cachemesh_metrics",
           [](Scheduler& s) {
             py::dict d;
             if (s.cachemesh() == nullptr) return d;
             const CacheMeshMetrics m = s.cachemesh()->metrics();
             d["l2_used"] = m.l2_used;
             d["l2_capacity"] = m.l2_capacity;
             d["l3_used"] = m.l3_used;
             d["l3_capacity"] = m.l3_capacity;
             d["offloads"] = m.offloads;
             d["l2_hits"] = m.l2_hits;
             d["l3_hits"] = m.l3_hits;
             d["misses"] = m.misses;
             d["l2_evictions"] = m.l2_evictions;
             d["l3_writes"] = m.l3_writes;
             d["l3_evictions"] = m.l3_evictions;
             return d;
           })
      .def("decode_candidates", &Scheduler::decode_candidates)
      .def("set_draft", &Scheduler::set_draft)
      .def("propose_ngram", &Scheduler::propose_ngram, py::arg("max_order") = 4, py::arg("min_order") = 1)
      .def("set_tail", &Scheduler::set_tail)
      .def("spec_stats",
           [](const Scheduler& s) {
             py::dict d;
             d["verify_groups"] = s.spec_steps();
             d["proposed"] = s.spec_proposed();
             d["accepted"] = s.spec_accepted();
             return d;
           })
      .def("kv_metrics", [](Scheduler& s) { return metrics_dict(s.blocks().metrics()); })
      .def("reset_prefix_cache", [](Scheduler& s) { s.blocks().reset_prefix_cache(); });

  register_cpu_ops(m);
  register_gguf(m);
  register_json(m);
  register_plugin(m);
  register_quantize(m);
  register_admission(m);
  register_schema(m);
  register_model_store(m);
  register_media_encode(m);
  register_image(m);
}
