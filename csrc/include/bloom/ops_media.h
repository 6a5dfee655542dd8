// Host entry points of the diffusion / media kernels (Wan 2.1 DiT, its VAE
// decoder and the umT5 text encoder), kept apart from ops.h so those
// translation units build on their own.
#pragma once
#include <torch/extension.h>

namespace bloom {

// csrc/kernels/wan.cu
void wan_residual_norm(torch::Tensor& x, const c10::optional<torch::Tensor>& delta,
                       const c10::optional<torch::Tensor>& gate_mod, const c10::optional<torch::Tensor>& gate_e,
                       int64_t gate_idx, int64_t gate_batch_stride, int64_t gate_idx_stride, int64_t mode, const c10::optional<torch::Tensor>& ln_w,
                       const c10::optional<torch::Tensor>& ln_b, const c10::optional<torch::Tensor>& mod,
                       const c10::optional<torch::Tensor>& e, int64_t shift_idx, int64_t scale_idx,
                       int64_t e_batch_stride, int64_t e_idx_stride, int64_t rows_per_batch, double eps,
                       torch::Tensor& y);
void wan_qkv_norm_rope(const torch::Tensor& src, int64_t q_col, int64_t k_col, int64_t v_col, int64_t heads,
                       int64_t head_dim, const c10::optional<torch::Tensor>& q_w,
                       const c10::optional<torch::Tensor>& k_w, double eps,
                       const c10::optional<torch::Tensor>& rope_tab, int64_t rope_pt, int64_t rope_ph,
                       int64_t grid_f, int64_t grid_h, int64_t grid_w, int64_t rows_per_batch,
                       const c10::optional<torch::Tensor>& q_out, const c10::optional<torch::Tensor>& kv,
                       int64_t blocks_per_batch, bool head_norm = false,
                       const c10::optional<torch::Tensor>& pos3 = c10::nullopt, int64_t out_rows_per_batch = 0,
                       int64_t out_offset = 0);
void wan_patchify(const torch::Tensor& latent, torch::Tensor& tokens);
void wan_unpatchify_step(const torch::Tensor& head_out, int64_t preds, double guidance, double dt,
                         torch::Tensor& latent);
void silu_bf16(const torch::Tensor& x, torch::Tensor& out);

// csrc/kernels/vae.cu
void vae_gn_stats(const torch::Tensor& x, int64_t groups, double eps, torch::Tensor& stats);
void vae_im2col3x3(const torch::Tensor& src, int64_t up, const c10::optional<torch::Tensor>& stats,
                   const c10::optional<torch::Tensor>& gamma, const c10::optional<torch::Tensor>& beta,
                   int64_t groups, bool silu, torch::Tensor& dst, int64_t stride = 1, int64_t pad_t = 1,
                   int64_t pad_b = 1, int64_t pad_l = 1, int64_t pad_r = 1);
void vae_gn_apply(const torch::Tensor& src, const torch::Tensor& stats, const torch::Tensor& gamma,
                  const torch::Tensor& beta, int64_t groups, bool silu, torch::Tensor& dst);
void vae_pack_attn(const torch::Tensor& qkv, int64_t frames, int64_t channels, torch::Tensor& q, torch::Tensor& kv);
void vae_rgb(const torch::Tensor& src, torch::Tensor& dst);

// csrc/kernels/t5.cu
void t5_rel_attention(const torch::Tensor& qkv, int64_t seqs, int64_t heads, const torch::Tensor& lens,
                      const torch::Tensor& bias, torch::Tensor& out);

}  // namespace bloom
