// End-to-end synthesis of one utterance: greedy MiniCPM-4 decode -> LocDiT CFM solve per step
// -> AudioVAE decode, mirroring the shape of VoxCpm2Model::inference (voxcpm2/model.rs:301-375)
// + VoxCPM::generate (voxcpm2/wrapper.rs:401-423) for this library's decode workload: the
// diffusion condition of step i is the base LM's final-norm hidden after decode step i (the
// reference feeds lm_to_dit_proj(lm_hidden) | res_to_dit_proj(residual_hidden), which needs
// the residual LM), the DiT prefix condition is the previous patch (zeros first), and the
// predicted patches are stacked [C, T*P] (stack_pred_feats, model.rs:283-287) for the VAE.
#include <vector>

#include "common.cuh"
#include "runtime.cuh"

using namespace vx;

extern "C" int vx_generate(vx_lm* lm, vx_dit* dit, vx_vae* vae, const int32_t* prompt_ids, int n_prompt,
                           const vx_generate_options* opts, const float* noise, float* wav_out, float* latent_out) {
  if (!lm || !dit || !vae || !prompt_ids || !opts || !noise || !wav_out || n_prompt <= 0) return VX_ERR_ARG;
  vx_ctx* ctx = lm_ctx(lm);
  if (dit_ctx(dit) != ctx || vae_ctx(vae) != ctx)
    return fail(ctx, VX_ERR_ARG, "generate: the LM, DiT and VAE must share one context");
  const int C = dit_in_channels(dit), P = opts->patch_size, n = opts->max_len, H = lm_hidden_size(lm);
  if (C != vae_latent(vae)) return fail(ctx, VX_ERR_CONFIG, "DiT channels %d != VAE latent %d", C, vae_latent(vae));
  if (P <= 0 || n <= 0 || opts->inference_timesteps < 1)
    return fail(ctx, VX_ERR_ARG, "generate: patch_size, max_len, inference_timesteps must be positive");
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  const size_t patch = (size_t)C * P, frames = (size_t)n * P, hop = vae_hop(vae);
  float *d_noise = nullptr, *d_cond = nullptr, *d_latent = nullptr, *d_wav = nullptr;
  auto cleanup = [&]() {
    for (float* p : {d_noise, d_cond, d_latent, d_wav})
      if (p) cudaFree(p);
  };
  if (cudaMalloc(&d_noise, patch * n * 4) != cudaSuccess || cudaMalloc(&d_cond, patch * 2 * 4) != cudaSuccess ||
      cudaMalloc(&d_latent, (size_t)C * frames * 4) != cudaSuccess ||
      cudaMalloc(&d_wav, frames * hop * 4) != cudaSuccess) {
    cudaGetLastError();
    cleanup();
    return fail(ctx, VX_ERR_OOM, "generate: buffer allocation failed");
  }
  int rc = VX_OK;
  do {
    if (cudaMemcpyAsync(d_noise, noise, patch * n * 4, cudaMemcpyDefault, st) != cudaSuccess ||
        cudaMemsetAsync(d_cond, 0, patch * 4, st) != cudaSuccess) {
      rc = fail(ctx, VX_ERR_CUDA, "generate: upload failed");
      break;
    }
    rc = lm_greedy_begin(lm, prompt_ids, n_prompt, n);
    if (rc) break;
    float* cond = d_cond;
    float* pred = d_cond + patch;
    for (int i = 0; i < n && !rc; ++i) {
      if (ctx->cancel.load(std::memory_order_relaxed)) {  // model.rs:330-334
        rc = fail(ctx, VX_ERR_CANCELLED, "generation cancelled");
        break;
      }
      rc = lm_greedy_step(lm);
      if (rc) break;
      // UnifiedCfm::forward(mu = hidden, cond = previous patch, z = noise_i) (model.rs:229-238)
      // queued without a host wait: the host runs ahead, the device never idles between steps
      rc = cfm_solve_enqueue(dit, lm_hid_norm(lm), cond, d_noise + patch * i, 1, H, P, P, opts->inference_timesteps,
                             opts->cfg_value, opts->sway_sampling_coef, opts->use_cfg_zero_star, pred);
      if (rc) break;
      // latent[:, i*P + p] = pred[:, p]
      if (cudaMemcpy2DAsync(d_latent + (size_t)i * P, frames * 4, pred, (size_t)P * 4, (size_t)P * 4, C,
                            cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
        rc = fail(ctx, VX_ERR_CUDA, "generate: latent stacking failed");
        break;
      }
      std::swap(cond, pred);  // the new patch conditions the next step (model.rs:241)
    }
    if (rc) break;
    rc = vx_vae_decode(vae, d_latent, 1, (int)frames, d_wav);
    if (rc) break;
    if (cudaMemcpyAsync(wav_out, d_wav, frames * hop * 4, cudaMemcpyDefault, st) != cudaSuccess ||
        (latent_out && cudaMemcpyAsync(latent_out, d_latent, (size_t)C * frames * 4, cudaMemcpyDefault, st) !=
                           cudaSuccess)) {
      rc = fail(ctx, VX_ERR_CUDA, "generate: download failed");
      break;
    }
    rc = vx_ctx_synchronize(ctx);
  } while (0);
  cudaStreamSynchronize(st);
  cleanup();
  return rc;
}

// B utterances in lockstep: one batched LM decode step (B rows) and one CFM solve over the B
// latents per patch, then one VAE decode of the B stacked latents.  Prompts share a length
// (a single device position); noise [B][max_len][C][P].
extern "C" int vx_generate_batch(vx_lm* lm, vx_dit* dit, vx_vae* vae, const int32_t* prompt_ids, int B, int n_prompt,
                                 const vx_generate_options* opts, const float* noise, float* wav_out,
                                 float* latent_out) {
  if (!lm || !dit || !vae || !prompt_ids || !opts || !noise || !wav_out || n_prompt <= 0 || B <= 0) return VX_ERR_ARG;
  vx_ctx* ctx = lm_ctx(lm);
  if (dit_ctx(dit) != ctx || vae_ctx(vae) != ctx)
    return fail(ctx, VX_ERR_ARG, "generate: the LM, DiT and VAE must share one context");
  const int C = dit_in_channels(dit), P = opts->patch_size, n = opts->max_len, H = lm_hidden_size(lm);
  if (C != vae_latent(vae)) return fail(ctx, VX_ERR_CONFIG, "DiT channels %d != VAE latent %d", C, vae_latent(vae));
  if (P <= 0 || n <= 0 || opts->inference_timesteps < 1)
    return fail(ctx, VX_ERR_ARG, "generate: patch_size, max_len, inference_timesteps must be positive");
  if (B > lm_max_batch(lm)) return fail(ctx, VX_ERR_SHAPE, "generate: %d utterances > the LM's max_batch", B);
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  const size_t patch = (size_t)C * P, frames = (size_t)n * P, hop = vae_hop(vae);
  float *d_noise = nullptr, *d_z = nullptr, *d_cond = nullptr, *d_latent = nullptr, *d_wav = nullptr;
  auto cleanup = [&]() {
    for (float* p : {d_noise, d_z, d_cond, d_latent, d_wav})
      if (p) cudaFree(p);
  };
  if (cudaMalloc(&d_noise, patch * n * B * 4) != cudaSuccess || cudaMalloc(&d_z, patch * B * 4) != cudaSuccess ||
      cudaMalloc(&d_cond, patch * 2 * B * 4) != cudaSuccess ||
      cudaMalloc(&d_latent, (size_t)C * frames * B * 4) != cudaSuccess ||
      cudaMalloc(&d_wav, frames * hop * B * 4) != cudaSuccess) {
    cudaGetLastError();
    cleanup();
    return fail(ctx, VX_ERR_OOM, "generate: buffer allocation failed");
  }
  int rc = VX_OK;
  do {
    if (cudaMemcpyAsync(d_noise, noise, patch * n * B * 4, cudaMemcpyDefault, st) != cudaSuccess ||
        cudaMemsetAsync(d_cond, 0, patch * B * 4, st) != cudaSuccess) {
      rc = fail(ctx, VX_ERR_CUDA, "generate: upload failed");
      break;
    }
    rc = lm_batch_begin(lm, prompt_ids, B, n_prompt, n);
    if (rc) break;
    float* cond = d_cond;
    float* pred = d_cond + patch * B;
    for (int i = 0; i < n && !rc; ++i) {
      if (ctx->cancel.load(std::memory_order_relaxed)) {  // model.rs:330-334
        rc = fail(ctx, VX_ERR_CANCELLED, "generation cancelled");
        break;
      }
      rc = lm_batch_step(lm);
      if (rc) break;
      // z_i of every utterance: noise[b][i] -> z [B, C, P]
      if (cudaMemcpy2DAsync(d_z, patch * 4, d_noise + patch * i, patch * n * 4, patch * 4, B, cudaMemcpyDeviceToDevice,
                            st) != cudaSuccess) {
        rc = fail(ctx, VX_ERR_CUDA, "generate: noise gather failed");
        break;
      }
      rc = cfm_solve_enqueue(dit, lm_batch_hidden(lm), cond, d_z, B, H, P, P, opts->inference_timesteps,
                             opts->cfg_value, opts->sway_sampling_coef, opts->use_cfg_zero_star, pred);
      if (rc) break;
      // latent[b][c][i*P + p] = pred[b][c][p]: B*C rows of P frames
      if (cudaMemcpy2DAsync(d_latent + (size_t)i * P, frames * 4, pred, (size_t)P * 4, (size_t)P * 4, (size_t)B * C,
                            cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
        rc = fail(ctx, VX_ERR_CUDA, "generate: latent stacking failed");
        break;
      }
      std::swap(cond, pred);
    }
    if (rc) break;
    rc = vx_vae_decode(vae, d_latent, B, (int)frames, d_wav);
    if (rc) break;
    if (cudaMemcpyAsync(wav_out, d_wav, frames * hop * B * 4, cudaMemcpyDefault, st) != cudaSuccess ||
        (latent_out && cudaMemcpyAsync(latent_out, d_latent, (size_t)C * frames * B * 4, cudaMemcpyDefault, st) !=
                           cudaSuccess)) {
      rc = fail(ctx, VX_ERR_CUDA, "generate: download failed");
      break;
    }
    rc = vx_ctx_synchronize(ctx);
  } while (0);
  cudaStreamSynchronize(st);
  cleanup();
  return rc;
}
