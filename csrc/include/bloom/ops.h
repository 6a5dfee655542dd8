// Host entry points of the bloom_b200._C extension (implemented in csrc/kernels/*.cu).
#pragma once

#include <torch/extension.h>

namespace bloom {

// GEMM epilogues (y = x @ w^T, w in nn.Linear layout [N, K]).
enum GemmEpilogue : int {
  kEpiBF16 = 0,        // out bf16 [M, N] (+bias)
  kEpiF32 = 1,         // out f32 [M, N] (+bias)
  kEpiSwiGLU = 2,      // w rows interleaved (16 gate | 16 up) per 32 rows; out bf16 [M, N/2] = silu(g) * u
  kEpiPartialF32 = 3,  // split-K: out f32 [splits, M, N] partial sums
  kEpiResidual = 4,    // out bf16 [M, N] = acc (+bias) + resid
  kEpiGelu = 5,        // out bf16 [M, N] = gelu_erf(acc + bias)
  kEpiGeluTanh = 6,    // out bf16 [M, N] = gelu_tanh(acc + bias) (runs the kEpiGelu kernels with Args::gelu_tanh)
  kEpiGeGLU = 7,       // as kEpiSwiGLU with gelu_tanh(g) * u (runs the kEpiSwiGLU kernels with Args::gelu_tanh)
};

// splits > 1 with a non-partial epilogue: split-K where the last-arriving CTA
// of each output tile sums the fp32 partials (fix_ws, L2-resident) and runs
// the fused epilogue; fix_count holds one self-resetting counter per tile.
void gemm_out(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, int64_t epi,
              const c10::optional<torch::Tensor>& resid, const c10::optional<torch::Tensor>& bias, int64_t splits,
              const torch::Tensor& status, const c10::optional<torch::Tensor>& fix_ws,
              const c10::optional<torch::Tensor>& fix_count, int64_t bn_override,
              const std::vector<int64_t>& push_ptrs = {}, int64_t push_rank = 0, int64_t push_rows = 0,
              int64_t wait_flags = 0, double wait_timeout_s = 5.0);
int64_t gemm_fixup_ws_floats(int64_t M, int64_t N, int64_t splits, int64_t bn_override);
int gemm_pick_bn(int M);
int gemm_default_splits(int M, int N, int K, int device);
void gemm_set_trace(const c10::optional<torch::Tensor>& buf);
void tp_ar_set_trace(const c10::optional<torch::Tensor>& buf);
void attn_tc_set_trace(const c10::optional<torch::Tensor>& buf);
int gemm_max_active_clusters(int64_t bn, int64_t cluster_size);

void gemm_grouped_out(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, int64_t epi,
                      const torch::Tensor& tiles, const torch::Tensor& num_tiles, int64_t rows_per_group, int64_t bn,
                      const torch::Tensor& status);

// Mixture of experts.
void moe_route(const torch::Tensor& logits, int64_t top_k, bool norm, int64_t e0, int64_t e_local,
               torch::Tensor& topk_ids, torch::Tensor& topk_w, torch::Tensor& slot, torch::Tensor& counts);
void moe_plan(torch::Tensor& counts, torch::Tensor& offsets, int64_t bn, int64_t ft_gu, int64_t ft_d,
              torch::Tensor& tiles_gu, torch::Tensor& n_gu, torch::Tensor& tiles_d, torch::Tensor& n_d);
void moe_gather(const torch::Tensor& x, int64_t e0, int64_t e_local, const torch::Tensor& topk_ids,
                const torch::Tensor& slot, const torch::Tensor& offsets, torch::Tensor& pos, torch::Tensor& xs);
void moe_combine(const torch::Tensor& ys, const torch::Tensor& pos, const torch::Tensor& topk_w, torch::Tensor& out,
                 const std::vector<int64_t>& push_ptrs = {}, int64_t push_rank = 0, int64_t push_rows = 0);

// Normalisation.
void rmsnorm(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& out, double eps);
// residual += sum_s delta[s] (delta is bf16 [M,H] or f32 [S,M,H]); out = rmsnorm(residual) * w
void add_rmsnorm(const torch::Tensor& delta, torch::Tensor& residual, const torch::Tensor& w, torch::Tensor& out,
                 double eps);
void layernorm(const torch::Tensor& x, const c10::optional<torch::Tensor>& resid, const torch::Tensor& w,
               const torch::Tensor& b, torch::Tensor& out, double eps);

// Embedding gather: out[t] = table[ids[t]] (rows outside [0, V) give zeros).
void embedding(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out);

// RoPE on q/k (+ optional per-head RMSNorm of q and k), q to q_out, k/v to the
// paged cache at slot_mapping (slot = block * 16 + offset; -1 skips).
void rope_kv_write(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& slot_mapping,
                   const torch::Tensor& cos_sin, torch::Tensor& q_out, torch::Tensor& kv_cache, int64_t layer,
                   int64_t num_q_heads, int64_t num_kv_heads, const c10::optional<torch::Tensor>& q_norm,
                   const c10::optional<torch::Tensor>& k_norm, double eps);

// Paged attention.
void paged_decode_attention(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                            const torch::Tensor& block_table, const torch::Tensor& seq_lens, torch::Tensor& out,
                            int64_t q_len, int64_t splits, torch::Tensor& workspace, double scale,
                            const torch::Tensor& status);
// int8 KV cache [L, NB, 2 x KVH x 16 x (128 + 4) bytes]: K pages, dim-major V pages, fp32 scales per block.
void paged_decode_attention_q8(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                               int64_t num_kv_heads, const torch::Tensor& block_table, const torch::Tensor& seq_lens,
                               torch::Tensor& out, int64_t q_len, int64_t splits, torch::Tensor& workspace,
                               double scale, const torch::Tensor& status);
void kv_dequant_pages_q8(const torch::Tensor& kv_cache, int64_t layer, int64_t num_kv_heads,
                         const torch::Tensor& block_table, const torch::Tensor& ctx_lens, int64_t W,
                         torch::Tensor& scratch, const torch::Tensor& status);
void rope_kv_write_q8(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& slot_mapping,
                      const torch::Tensor& cos_sin, torch::Tensor& q_out, torch::Tensor& kv_cache, int64_t layer,
                      int64_t num_q_heads, int64_t num_kv_heads, const c10::optional<torch::Tensor>& q_norm,
                      const c10::optional<torch::Tensor>& k_norm, double eps);
void paged_prefill_attention(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                             const torch::Tensor& block_table, const torch::Tensor& ctx_lens,
                             const torch::Tensor& cu_seqlens_q, const torch::Tensor& tile_seq,
                             const torch::Tensor& tile_start, torch::Tensor& out, double scale, bool causal,
                             const torch::Tensor& status);
// Same contract on tcgen05 (S and O in TMEM), head_dim 128, 128-row tiles
// (tile_start in steps of 128 within a sequence).
void paged_prefill_attention_tc(const torch::Tensor& q, const torch::Tensor& kv_cache, int64_t layer,
                                const torch::Tensor& block_table, const torch::Tensor& ctx_lens,
                                const torch::Tensor& cu_seqlens_q, const torch::Tensor& tile_seq,
                                const torch::Tensor& tile_start, torch::Tensor& out, double scale, bool causal,
                                const torch::Tensor& status);
int64_t decode_attention_splits(int64_t batch, int64_t num_kv_heads, int64_t max_pages, int64_t device);
// CTAs per KV head for decode/verify attention: the smallest divisor hc of
// G = q heads per KV head with (G / hc) * q_len <= 32 (0 if none).
int64_t decode_head_chunks(int64_t num_q_heads, int64_t num_kv_heads, int64_t q_len);

// Sampling.
void argmax_rows(const torch::Tensor& logits, torch::Tensor& out);
void apply_token_mask(torch::Tensor& logits, const torch::Tensor& rows, const torch::Tensor& mask, int64_t col_offset);
void sample_rows(const torch::Tensor& logits, const torch::Tensor& temperature, const torch::Tensor& top_p,
                 const torch::Tensor& top_k, const torch::Tensor& seeds, const torch::Tensor& offsets,
                 torch::Tensor& out);
// Sampling with speculative verification.  Row b carries a proposal
// draft[b] (-1: none).  Greedy rows return the argmax.  Stochastic rows accept
// the proposal with probability p(draft) under the row's temperature/top-k/
// top-p distribution, otherwise draw from that distribution with the proposal
// removed (rejection sampling with a deterministic proposal; exact for the
// target distribution).  A row without a proposal samples as sample_rows.
// GGUF Q8_0 (kind 0) / Q4_0 (kind 1) weights kept quantised on the device
// (quant plane + fp16 scale plane [N, K/32]).  qgemv: M <= 8 tokens with a
// bf16, SwiGLU (interleaved rows) or residual epilogue; qdequant: bf16 [N, K].
void qgemv(const torch::Tensor& x, const torch::Tensor& qs, const torch::Tensor& scales, int64_t kind,
           torch::Tensor& out, int64_t epi, const c10::optional<torch::Tensor>& resid);
void qdequant(const torch::Tensor& qs, const torch::Tensor& scales, int64_t kind, torch::Tensor& out);

// Non-GGUF weight formats and 8-bit KV rows (quant_formats.cu).
void int4_flat_dequant(const torch::Tensor& qweight, const torch::Tensor& scales, const torch::Tensor& qzeros,
                       const c10::optional<torch::Tensor>& g_idx, torch::Tensor& out);
void gptq_dequant(const torch::Tensor& qweight, const torch::Tensor& qzeros, const torch::Tensor& scales,
                  const torch::Tensor& g_idx, torch::Tensor& out);
void awq_dequant(const torch::Tensor& qweight, const torch::Tensor& qzeros, const torch::Tensor& scales,
                 int64_t group, torch::Tensor& out);
void bnb4_dequant(const torch::Tensor& packed, const torch::Tensor& scale, int64_t block, bool nf4,
                  torch::Tensor& out);
void kv_row_quant(const torch::Tensor& x, torch::Tensor& q, torch::Tensor& scales, bool fp8);
void kv_row_dequant(const torch::Tensor& q, const torch::Tensor& scales, torch::Tensor& out, bool fp8);

// Multimodal rotary embedding (mrope.cu): cos / sin fp32 [3, B, S, D].
void mrope(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& cos, const torch::Tensor& sin,
           torch::Tensor& q_out, torch::Tensor& k_out, int64_t sec0, int64_t sec1, int64_t sec2);

void verify_sample_rows(const torch::Tensor& logits, const torch::Tensor& temperature, const torch::Tensor& top_p,
                        const torch::Tensor& top_k, const torch::Tensor& seeds, const torch::Tensor& offsets,
                        const torch::Tensor& draft, torch::Tensor& out);

// Tensor-parallel collectives over peer memory (pointers are device addresses
// valid in this process, one per rank: the local buffer and the peer mappings).
int64_t tp_flag_words();
void tp_allreduce_rmsnorm(const std::vector<int64_t>& partial_ptrs, const std::vector<int64_t>& x_ptrs,
                          const std::vector<int64_t>& flag_ptrs, int64_t rank, torch::Tensor& residual,
                          const torch::Tensor& w, double eps, int64_t T, double timeout_s,
                          const torch::Tensor& status, bool pushed = false, bool defer_done = false);
void tp_allgather_rows(const torch::Tensor& src, const std::vector<int64_t>& dst_ptrs,
                       const std::vector<int64_t>& flag_ptrs, int64_t rank, int64_t T, double timeout_s,
                       const torch::Tensor& status);
void tp_barrier(const std::vector<int64_t>& flag_ptrs, int64_t rank, double timeout_s, const torch::Tensor& status);
void tp_argmax_gather(const torch::Tensor& logits, int64_t vocab_offset, const std::vector<int64_t>& slot_ptrs,
                      int64_t max_rows, const std::vector<int64_t>& flag_ptrs, int64_t rank, torch::Tensor& out,
                      double timeout_s, const torch::Tensor& status);
void tp_gather_cols(const torch::Tensor& logits, const std::vector<int64_t>& dst_ptrs, int64_t dst_cols,
                    const std::vector<int64_t>& stat_ptrs, const std::vector<int64_t>& flag_ptrs, int64_t rank,
                    torch::Tensor& out_status, double timeout_s, const torch::Tensor& status);

// Encoder (BERT) kernels.
void bert_embed_ln(const torch::Tensor& ids, const torch::Tensor& pos, const c10::optional<torch::Tensor>& types,
                   const torch::Tensor& word, const torch::Tensor& pemb, const torch::Tensor& temb,
                   const torch::Tensor& g, const torch::Tensor& b, torch::Tensor& out, double eps);
void varlen_attention(const torch::Tensor& qkv, const torch::Tensor& cu_seqlens, torch::Tensor& out, int64_t num_heads,
                      int64_t head_dim, int64_t max_len, double scale);
void mean_pool_l2(const torch::Tensor& x, const torch::Tensor& cu_seqlens, torch::Tensor& out, bool normalize);
void ln_residual_f32(const torch::Tensor& delta, const torch::Tensor& resid, const torch::Tensor& g,
                     const torch::Tensor& b, torch::Tensor& out, double eps);
void gelu_f32_(torch::Tensor& x);

// Status word.
torch::Tensor status_tensor(int64_t device);
// Status word for kernels' index checks: only builds with -DBLOOM_KERNEL_CHECKS
// pass one (the regular build passes nullptr and its kernels never look).
inline int* check_word(int64_t device) {
#ifdef BLOOM_KERNEL_CHECKS
  return status_tensor(device).data_ptr<int>();
#else
  (void)device;
  return nullptr;
#endif
}

// Gemma4 (csrc/kernels/gemma.cu): wide-head paged attention with sliding windows and
// soft-capping, q/k/v norm + partial RoPE + KV write, sandwich residual norms, logit soft-cap
int64_t wide_decode_splits(int64_t batch, int64_t nq, int64_t nkv, int64_t head_dim, int64_t q_len,
                           int64_t max_kv_len, int64_t window, int64_t num_sms);
int64_t wide_decode_workspace_numel(int64_t batch, int64_t nq, int64_t nkv, int64_t head_dim, int64_t q_len,
                                    int64_t splits);
void wide_decode_attention(const torch::Tensor& q, torch::Tensor& out, const torch::Tensor& kv_layer, int64_t nkv,
                           const torch::Tensor& block_table, const torch::Tensor& seq_lens, int64_t q_len,
                           int64_t window, double scale, double softcap, int64_t splits,
                           const c10::optional<torch::Tensor>& workspace, const torch::Tensor& status);
void wide_prefill_attention(const torch::Tensor& q, torch::Tensor& out, const torch::Tensor& kv_layer, int64_t nkv,
                            const torch::Tensor& block_table, const torch::Tensor& ctx_lens,
                            const torch::Tensor& cu_q, const torch::Tensor& tile_seq,
                            const torch::Tensor& tile_start, int64_t window, double scale, double softcap,
                            const torch::Tensor& status, bool causal = true);
void gemma_qkv_write(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& slots,
                     const torch::Tensor& cos_sin, torch::Tensor& q_out, torch::Tensor& kv_layer, int64_t nq,
                     int64_t nkv, int64_t rot, const torch::Tensor& q_w, const torch::Tensor& k_w, double eps,
                     bool k_eq_v, const torch::Tensor& status);
void residual_norm(const torch::Tensor& a, torch::Tensor& x, const c10::optional<torch::Tensor>& w_post,
                   const c10::optional<torch::Tensor>& w_next, const c10::optional<torch::Tensor>& y,
                   double in_scale, double out_scale, double eps);
void softcap_(torch::Tensor& v, double cap);

}  // namespace bloom
