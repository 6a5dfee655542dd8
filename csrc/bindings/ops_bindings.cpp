// pybind11 surface of bloom_b200._C (CUDA kernels for sm_100a).
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "bloom/ops.h"
#include "bloom/ops_media.h"

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "bloom_b200 sm_100a kernels";
#ifdef BLOOM_KERNEL_CHECKS
  m.attr("KERNEL_CHECKS") = true;
#else
  m.attr("KERNEL_CHECKS") = false;
#endif
  m.attr("STATUS_INDEX_CHECK") = 1 << 6;  // kStatusIndexCheck in bloom/common.cuh
  m.attr("EPI_BF16") = int(bloom::kEpiBF16);
  m.attr("EPI_F32") = int(bloom::kEpiF32);
  m.attr("EPI_SWIGLU") = int(bloom::kEpiSwiGLU);
  m.attr("EPI_PARTIAL_F32") = int(bloom::kEpiPartialF32);
  m.attr("EPI_RESIDUAL") = int(bloom::kEpiResidual);
  m.attr("EPI_GELU") = int(bloom::kEpiGelu);
  m.attr("EPI_GEGLU") = int(bloom::kEpiGeGLU);
  m.def("gemm_out", &bloom::gemm_out, "y = x @ w^T on tcgen05 with fused epilogue", py::arg("x"), py::arg("w"),
        py::arg("out"), py::arg("epi"), py::arg("resid"), py::arg("bias"), py::arg("splits"), py::arg("status"),
        py::arg("fix_ws"), py::arg("fix_count"), py::arg("bn_override"),
        py::arg("push_ptrs") = std::vector<int64_t>{}, py::arg("push_rank") = 0, py::arg("push_rows") = 0,
        py::arg("wait_flags") = 0, py::arg("wait_timeout_s") = 5.0);
  m.def("gemm_pick_bn", &bloom::gemm_pick_bn);
  m.def("gemm_grouped_out", &bloom::gemm_grouped_out);
  m.def("moe_route", &bloom::moe_route);
  m.def("moe_plan", &bloom::moe_plan);
  m.def("wide_decode_splits", &bloom::wide_decode_splits);
  m.def("wide_decode_workspace_numel", &bloom::wide_decode_workspace_numel);
  m.def("wide_decode_attention", &bloom::wide_decode_attention);
  m.def("wide_prefill_attention", &bloom::wide_prefill_attention, py::arg("q"), py::arg("out"), py::arg("kv_layer"),
        py::arg("nkv"), py::arg("block_table"), py::arg("ctx_lens"), py::arg("cu_q"), py::arg("tile_seq"),
        py::arg("tile_start"), py::arg("window"), py::arg("scale"), py::arg("softcap"), py::arg("status"),
        py::arg("causal") = true);
  m.def("gemma_qkv_write", &bloom::gemma_qkv_write);
  m.def("residual_norm", &bloom::residual_norm);
  m.def("softcap_", &bloom::softcap_);
  m.def("wan_residual_norm", &bloom::wan_residual_norm);
  m.def("wan_qkv_norm_rope", &bloom::wan_qkv_norm_rope, py::arg("src"), py::arg("q_col"), py::arg("k_col"),
        py::arg("v_col"), py::arg("heads"), py::arg("head_dim"), py::arg("q_w"), py::arg("k_w"), py::arg("eps"),
        py::arg("rope_tab"), py::arg("rope_pt"), py::arg("rope_ph"), py::arg("grid_f"), py::arg("grid_h"),
        py::arg("grid_w"), py::arg("rows_per_batch"), py::arg("q_out"), py::arg("kv"), py::arg("blocks_per_batch"),
        py::arg("head_norm") = false, py::arg("pos3") = py::none(), py::arg("out_rows_per_batch") = 0,
        py::arg("out_offset") = 0);
  m.def("wan_patchify", &bloom::wan_patchify);
  m.def("wan_unpatchify_step", &bloom::wan_unpatchify_step);
  m.def("silu_bf16", &bloom::silu_bf16);
  m.def("vae_gn_stats", &bloom::vae_gn_stats);
  m.def("vae_im2col3x3", &bloom::vae_im2col3x3, py::arg("src"), py::arg("up"), py::arg("stats"), py::arg("gamma"),
        py::arg("beta"), py::arg("groups"), py::arg("silu"), py::arg("dst"), py::arg("stride") = 1,
        py::arg("pad_t") = 1, py::arg("pad_b") = 1, py::arg("pad_l") = 1, py::arg("pad_r") = 1);
  m.def("vae_gn_apply", &bloom::vae_gn_apply);
  m.def("vae_pack_attn", &bloom::vae_pack_attn);
  m.def("vae_rgb", &bloom::vae_rgb);
  m.def("t5_rel_attention", &bloom::t5_rel_attention);
  m.def("moe_gather", &bloom::moe_gather);
  m.def("moe_combine", &bloom::moe_combine, py::arg("ys"), py::arg("pos"), py::arg("topk_w"), py::arg("out"),
        py::arg("push_ptrs") = std::vector<int64_t>{}, py::arg("push_rank") = 0, py::arg("push_rows") = 0);
  m.def("gemm_default_splits", &bloom::gemm_default_splits);
  m.def("gemm_max_active_clusters", &bloom::gemm_max_active_clusters, "resident clusters of the one-CTA GEMM");
  m.def("attn_tc_set_trace", &bloom::attn_tc_set_trace, "per-CTA phase profile of tcgen05 prefill launches (None = off)");
  m.def("tp_ar_set_trace", &bloom::tp_ar_set_trace, "phase timeline of tp_allreduce_rmsnorm block 0 (None = off)");
  m.def("gemm_set_trace", &bloom::gemm_set_trace, "per-CTA %globaltimer timeline of plain GEMM launches (None = off)");
  m.def("gemm_fixup_ws_floats", &bloom::gemm_fixup_ws_floats);
  m.def("rmsnorm", &bloom::rmsnorm);
  m.def("add_rmsnorm", &bloom::add_rmsnorm);
  m.def("layernorm", &bloom::layernorm);
  m.def("embedding", &bloom::embedding);
  m.def("rope_kv_write", &bloom::rope_kv_write);
  m.def("paged_decode_attention", &bloom::paged_decode_attention);
  m.def("paged_prefill_attention", &bloom::paged_prefill_attention);
  m.def("decode_attention_splits", &bloom::decode_attention_splits);
  m.def("decode_head_chunks", &bloom::decode_head_chunks);
  m.def("paged_prefill_attention_tc", &bloom::paged_prefill_attention_tc);
  m.def("argmax_rows", &bloom::argmax_rows);
  m.def("apply_token_mask", &bloom::apply_token_mask);
  m.def("sample_rows", &bloom::sample_rows);
  m.def("verify_sample_rows", &bloom::verify_sample_rows);
  m.def("qgemv", &bloom::qgemv, py::arg("x"), py::arg("qs"), py::arg("scales"), py::arg("kind"), py::arg("out"),
        py::arg("epi"), py::arg("resid") = py::none());
  m.def("qdequant", &bloom::qdequant);
  m.def("int4_flat_dequant", &bloom::int4_flat_dequant, py::arg("qweight"), py::arg("scales"), py::arg("qzeros"),
        py::arg("g_idx"), py::arg("out"), "AWQ (g_idx None) / GPTQ int4 in the flat layout");
  m.def("gptq_dequant", &bloom::gptq_dequant, "GPTQ checkpoint tensors -> W [N, K] bf16");
  m.def("awq_dequant", &bloom::awq_dequant, "AWQ GEMM-format checkpoint tensors -> W [N, K] bf16");
  m.def("bnb4_dequant", &bloom::bnb4_dequant, "bitsandbytes NF4 / FP4 codes -> bf16");
  m.def("kv_row_quant", &bloom::kv_row_quant, "per-row int8 / e4m3 quantisation");
  m.def("kv_row_dequant", &bloom::kv_row_dequant, "per-row int8 / e4m3 dequantisation");
  m.def("mrope", &bloom::mrope, "multimodal rotary embedding on q [B,H,S,D], k [B,KVH,S,D]");
  m.def("status_tensor", &bloom::status_tensor);
  m.def("bert_embed_ln", &bloom::bert_embed_ln);
  m.def("varlen_attention", &bloom::varlen_attention);
  m.def("ln_residual_f32", &bloom::ln_residual_f32);
  m.def("gelu_f32_", &bloom::gelu_f32_);
  m.def("paged_decode_attention_q8", &bloom::paged_decode_attention_q8);
  m.def("kv_dequant_pages_q8", &bloom::kv_dequant_pages_q8);
  m.def("rope_kv_write_q8", &bloom::rope_kv_write_q8);
  m.def("mean_pool_l2", &bloom::mean_pool_l2);
  m.def("tp_flag_words", &bloom::tp_flag_words);
  m.def("tp_allreduce_rmsnorm", &bloom::tp_allreduce_rmsnorm, py::arg("partial_ptrs"), py::arg("x_ptrs"),
        py::arg("flag_ptrs"), py::arg("rank"), py::arg("residual"), py::arg("w"), py::arg("eps"), py::arg("T"),
        py::arg("timeout_s"), py::arg("status"), py::arg("pushed") = false, py::arg("defer_done") = false);
  m.def("tp_allgather_rows", &bloom::tp_allgather_rows);
  m.def("tp_barrier", &bloom::tp_barrier);
  m.def("tp_argmax_gather", &bloom::tp_argmax_gather);
  m.def("tp_gather_cols", &bloom::tp_gather_cols);
}
