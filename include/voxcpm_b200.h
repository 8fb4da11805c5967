/*
 * voxcpm_b200.h -- C ABI of libvoxcpm_b200.so, the B200 (sm_100a) implementation of the
 * voxcpm-rs hot path: the MiniCPM-4 decode step, the LocDiT flow-matching step and the
 * AudioVAE decoder.
 *
 * Conventions
 *   - Every function returns a vx_status (0 = VX_OK).  On failure vx_last_error(ctx) holds
 *     a message.  No function aborts; kernels never trap (bounded device waits report
 *     VX_ERR_TIMEOUT instead).
 *   - Op-level calls take caller-owned DEVICE pointers and run on `stream` (a cudaStream_t;
 *     NULL = the legacy default stream, as in cuBLAS; pass vx_ctx_stream(ctx) for the
 *     context's own stream).  They are asynchronous with respect to the host.
 *   - Model objects (vx_lm, vx_dit, vx_vae) own their weights, KV caches and work buffers.
 *     Weight loads accept host or device pointers (copied with cudaMemcpyDefault), bf16
 *     weights as raw bit patterns (uint16_t) in the checkpoint's [out, in] layout.
 *   - Threading mirrors the reference's !Sync model (README.md:96-103): one host thread per
 *     context.  vx_cancel is the only call that is safe from another thread.
 *
 * Reference citations are paths inside the voxcpm-rs crate.
 */
#ifndef VOXCPM_B200_H
#define VOXCPM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes mirror src/error.rs:7-55 where a counterpart exists. */
typedef enum {
  VX_OK = 0,
  VX_ERR_SHAPE = 1,     /* Error::ShapeMismatch (error.rs:36-41) */
  VX_ERR_CONFIG = 2,    /* Error::InvalidConfig (error.rs:30-31) */
  VX_ERR_CANCELLED = 3, /* Error::Cancelled (error.rs:49-51) */
  VX_ERR_KV_FULL = 4,   /* the `KV cache is full` assert (minicpm4/cache.rs:61) */
  VX_ERR_CUDA = 5,      /* a CUDA runtime error */
  VX_ERR_TIMEOUT = 6,   /* a bounded device-side wait gave up */
  VX_ERR_ARG = 7,       /* null pointer / invalid argument */
  VX_ERR_OOM = 8,       /* device allocation failed */
  VX_ERR_NO_DEVICE = 9  /* no usable CUDA device */
} vx_status;

typedef struct vx_ctx vx_ctx;
typedef struct vx_lm vx_lm;
typedef struct vx_dit vx_dit;
typedef struct vx_vae vx_vae;
typedef struct vx_vae_stream vx_vae_stream;
typedef void* vx_stream;

/* MiniCpm4Config + RopeScalingConfig (src/config.rs:42-84).  Factor arrays are host
 * pointers of rope_factor_len floats (= head_dim/2, asserted as in minicpm4/rope.rs:32). */
typedef struct {
  int hidden_size;
  int intermediate_size;
  int num_attention_heads;
  int num_key_value_heads;
  int num_hidden_layers;
  int vocab_size;
  int kv_channels; /* 0 = hidden_size / num_attention_heads */
  int max_position_embeddings;
  int original_max_position_embeddings;
  float rms_norm_eps;
  float rope_theta;
  int use_mup;
  float scale_emb;
  float scale_depth;
  int no_rope;
  const float* rope_short_factor;
  const float* rope_long_factor;
  int rope_factor_len;
} vx_minicpm4_config;

/* ----------------------------------------------------------------- context */

/* Library version (major*10000 + minor*100 + patch). */
int vx_version(void);
/* Number of CUDA kernels the calling thread has launched through this library (a graph
 * replay counts the kernels it holds).  No reference counterpart: instrumentation. */
unsigned long long vx_launch_count(void);
/* Create a context bound to CUDA device `device` (its own stream, scratch pool). */
int vx_ctx_create(int device, vx_ctx** out);
void vx_ctx_destroy(vx_ctx* ctx);
/* Message for the last failed call on this context (never NULL). */
const char* vx_last_error(const vx_ctx* ctx);
/* The context's cudaStream_t. */
void* vx_ctx_stream(vx_ctx* ctx);
/* Wait for the context's stream; reports VX_ERR_TIMEOUT if a device wait gave up. */
int vx_ctx_synchronize(vx_ctx* ctx);
/* CancelToken::cancel (voxcpm2/wrapper.rs:57-59): thread-safe; polled between AR steps
 * (voxcpm2/model.rs:330-334). */
void vx_cancel(vx_ctx* ctx);
/* Clear the cancel flag (a fresh CancelToken). */
void vx_cancel_reset(vx_ctx* ctx);
/* Copy `bytes` between any two host/device pointers on the context's stream, then wait. */
int vx_memcpy(vx_ctx* ctx, void* dst, const void* src, size_t bytes);

/* ----------------------------------------------------------------- ops */

/* MiniCpmDecoderLayer::add_residual (minicpm4/layer.rs:33-38) fused with
 * MiniCpmRmsNorm::forward (minicpm4/mod.rs:54-68):
 *   h = r + x * resid_scale   (r may be NULL: h = x)
 *   y = h * (mean(h^2) + eps)^-1/2 * w
 * x, r, h_out, y_out: [rows, hidden] f32; w: [hidden] f32.  h_out may be NULL. */
int vx_rmsnorm_residual(vx_ctx* ctx, const float* x, const float* r, const float* w, float resid_scale,
                        float eps, int rows, int hidden, float* h_out, float* y_out, vx_stream stream);

/* MiniCpmLongRope::new (minicpm4/rope.rs:16-54), host-side: rows 0..n_pos of the f64-built
 * cos/sin tables rounded to f32, each [n_pos, head_dim] (host pointers). */
int vx_longrope_table(const vx_minicpm4_config* cfg, int n_pos, float* cos_out, float* sin_out);

/* apply_rotary_pos_emb (minicpm4/rope.rs:76-95), in place on q [B,nh,S,d] and k [B,nkv,S,d]
 * with gathered cos/sin rows [S, d] (MiniCpmLongRope::gather, rope.rs:58-62). */
int vx_rope_apply(vx_ctx* ctx, float* q, float* k, const float* cos, const float* sin, int B, int nh, int nkv,
                  int S, int head_dim, vx_stream stream);

/* burn::nn::Linear::forward with bf16 weights [N, K] ([out, in]) and optional bias [N]:
 * y[M, N] = x[M, K] . W^T + b.  M = 1 uses the streamed GEMV. */
int vx_linear_bf16(vx_ctx* ctx, const uint16_t* w, const float* bias, const float* x, int M, int N, int K,
                   float* y, vx_stream stream);

/* MiniCpmAttention::sdpa + repeat_kv over a static cache (minicpm4/attention.rs:129-150,
 * 156-204) for one query token per batch row: q [B, nh*d], caches [B, nkv, s_max, d] filled
 * over 0..cur_len, out [B, nh*d].  Split-K flash-decode; uses context scratch memory. */
int vx_attention_decode(vx_ctx* ctx, const float* q, const float* kcache, const float* vcache, int B, int nh,
                        int nkv, int head_dim, int s_max, int cur_len, float* out, vx_stream stream);

/* vx_attention_decode for callers that cannot allocate device memory (a host that gives
 * the library a fixed memory budget, or a real-time thread where a cudaMalloc could stall
 * the device): no context, no allocation of any kind.  Its scratch is a file-scope device
 * array of 1 MiB plus 64 counters, held by every GPU that loads the library until exit, so
 * it accepts B * nkv <= 64 and B * nkv * 16 * 8 * (head_dim + 2) * 4 <= 1 MiB (else
 * VX_ERR_SHAPE).  The first call on a device looks up the array's device address; make that
 * call before any stream capture.  The address is kept for the life of the process: it does
 * not survive cudaDeviceReset, so do not call this after resetting a device the library has
 * already used.  All calls share the array: calls that overlap on the GPU
 * race and must be serialised by the caller.  Returns a status code only (no context, so no
 * message).  Same arguments and results as vx_attention_decode; `stream` NULL = the legacy
 * default stream.  No counterpart in the reference. */
int vx_attention_decode_static(const float* q, const float* kcache, const float* vcache, int B, int nh, int nkv,
                               int head_dim, int s_max, int cur_len, float* out, vx_stream stream);

/* MiniCpmMlp::forward (minicpm4/mlp.rs:28-34): out = down(silu(gate) * up) with the fused
 * gate|up weight [2*inter, hidden] (gate first) and down [hidden, inter]; x [rows, hidden]. */
int vx_mlp_swiglu(vx_ctx* ctx, const uint16_t* w_gate_up, const uint16_t* w_down, const float* x, int rows,
                  int hidden, int inter, float* out, vx_stream stream);

/* UnifiedCfm::solve_euler's per-step update (locdit/unified_cfm.rs:132-158), fused:
 * out2b [2B, C, T] holds the conditional rows then the unconditional rows of the DiT
 * output; x [B, C, T] is updated in place: x -= dt * v, with v the CFG or CFG-zero-star
 * velocity at guidance `cfg`. */
int vx_cfg_euler(vx_ctx* ctx, const float* out2b, float* x, int B, int C, int T, float cfg, double dt,
                 int zero_star, vx_stream stream);

/* ScalarQuantizationLayer::forward (fsq.rs:24-29): out = out_proj(round(tanh(in_proj(h)) *
 * scale) / scale), in_proj / out_proj Linears with bias (bf16 weights in the checkpoint's
 * [out, in] layout, f32 biases; biases may be NULL).  h [rows, in_dim] -> out [rows, out_dim];
 * latent_dim is in_proj's width.  Rounding is half away from zero (Rust f32::round). */
int vx_fsq(vx_ctx* ctx, const uint16_t* w_in, const float* b_in, const uint16_t* w_out, const float* b_out,
           int in_dim, int latent_dim, int out_dim, float scale, const float* hidden, int rows, float* out,
           vx_stream stream);

/* ----------------------------------------------------------------- MiniCPM-4 model */

/* MiniCpmModel::new (minicpm4/model.rs:26-41) + StaticKvCache::new (minicpm4/cache.rs:21-44)
 * for up to max_batch rows and max_length positions. */
int vx_lm_create(vx_ctx* ctx, const vx_minicpm4_config* cfg, int max_batch, int max_length, vx_lm** out);
void vx_lm_destroy(vx_lm* lm);
/* One decoder layer's weights in checkpoint layout; q/k/v and gate/up are fused on upload
 * as weights.rs:648-772 does. */
int vx_lm_load_layer(vx_lm* lm, int layer, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                     const uint16_t* o, const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                     const float* ln_in, const float* ln_post);
int vx_lm_load_norm(vx_lm* lm, const float* w);
/* Tied token embedding [vocab, hidden] bf16 (Embedding in minicpm4/model.rs:27-28). */
int vx_lm_load_embed(vx_lm* lm, const uint16_t* embed);
/* StaticKvCache::reset (minicpm4/cache.rs:67-69). */
int vx_lm_reset(vx_lm* lm);
/* StaticKvCache::current_length. */
int vx_lm_position(const vx_lm* lm);
int vx_lm_set_position(vx_lm* lm, int pos);
/* Write / read positions 0..n_pos of one layer's K and V cache for batch row `b`
 * ([nkv, n_pos, d] f32 each, host or device pointers). */
int vx_lm_kv_write(vx_lm* lm, int layer, int b, const float* k, const float* v, int n_pos);
int vx_lm_kv_read(vx_lm* lm, int layer, int b, float* k, float* v, int n_pos);
/* MiniCpmModel::embed * scale_emb (minicpm4/model.rs:87-100): ids [n] device int32,
 * out [n, hidden] device. */
int vx_lm_embed(vx_lm* lm, const int32_t* ids, int n, float* out);
/* MiniCpmModel::forward (minicpm4/model.rs:43-62): embeds/hidden_out [B, S, hidden] device.
 * With fill_cache the post-RoPE K/V of positions 0..S seed the cache and the position
 * becomes S (StaticKvCache::fill, cache.rs:47-58). */
int vx_lm_forward(vx_lm* lm, const float* embeds, int B, int S, int causal, int fill_cache, float* hidden_out);
/* MiniCpmModel::forward_step (minicpm4/model.rs:64-84) for batch 1: takes the position from
 * StaticKvCache::step (cache.rs:60-65; VX_ERR_KV_FULL when full).  embeds/hidden_out [hidden]. */
int vx_lm_forward_step(vx_lm* lm, const float* embeds, float* hidden_out);
/* MiniCpmDecoderLayer::forward_step (minicpm4/layer.rs:57-73) for batch 1 at position `pos`,
 * in place on hidden [hidden] (device). */
int vx_lm_layer_forward_step(vx_lm* lm, int layer, float* hidden, int pos);
/* Greedy decode over the tied embedding (the LM-decode workload; the reference has no LM
 * head): causal prefill of the prompt (host int32 ids) filling the cache, then n_steps
 * forward_step calls.  Each pick is argmax(norm(h) . E^T) (ties -> lowest id) and feeds
 * embed(id) * scale_emb back.  tokens_out (host) receives n_steps + 1 ids (the first from the
 * prefill's last row).  The decode step runs as one captured CUDA graph replayed per step
 * with no host round trip; cancellation (vx_cancel) is polled between steps. */
int vx_lm_greedy(vx_lm* lm, const int32_t* prompt_ids, int n_prompt, int n_steps, int32_t* tokens_out);
/* One batch-1 decode step at `pos` run eagerly (no graph, no programmatic dependent launch)
 * with a CUDA event after every kernel: kernel_us receives num_hidden_layers*5 + 1 durations
 * (per layer: qkv+rope, attention, o_proj, gate_up, down; then the greedy head).  Writes the
 * KV cache at `pos` and does not advance the position.  Instrumentation, no reference
 * counterpart beyond the VOXCPM_PROFILE timing split (voxcpm2/model.rs:316-372). */
int vx_lm_profile_decode_step(vx_lm* lm, int pos, float* kernel_us, int n);
/* One persistent decode step (the single-launch form vx_lm_greedy replays) at `pos` with its
 * phase trace on.  trace_out (host, n >= (num_hidden_layers*4 + 1) * grid * 8 entries)
 * receives, per phase p (qkv+rope, attention, o_proj, MLP per layer; then the head) and
 * CTA c, the %globaltimer ns at [(p*grid + c)*8 + k]: k = 0 phase start, 1 inputs ready,
 * 2 phase published, 3 first operand copy issued, 4 last copy issued, 5 last unit computed,
 * 6 first stage available, 7 first unit computed (0 where the CTA had no work).
 * *grid_out receives the grid.  Advances the position and greedy step
 * like a replayed step.  VX_ERR_CONFIG when the model runs the per-kernel step.
 * Instrumentation, no reference counterpart. */
int vx_lm_trace_decode_step(vx_lm* lm, int pos, unsigned long long* trace_out, int n, int* grid_out);
/* Device time of the last vx_lm_greedy call split into prefill and decode (CUDA events on
 * the context stream).  Mirrors the VOXCPM_PROFILE split of voxcpm2/model.rs:316-372. */
int vx_lm_last_timing(const vx_lm* lm, float* prefill_ms, float* decode_ms);
/* Logits of the last greedy pick (host [vocab]); valid after vx_lm_greedy. */
int vx_lm_last_logits(vx_lm* lm, float* logits_out);

/* ----------------------------------------------------------------- LocDiT + CFM */

/* VoxCpmLocDiTV2::new (locdit/local_dit.rs:83-96): the DiT decoder is a MiniCPM-4 built from
 * `cfg` (vocab_size must be 0, as asserted at local_dit.rs:84); max_rows bounds the batch of
 * DiT rows (2B for a CFG solve of B latents). */
int vx_dit_create(vx_ctx* ctx, const vx_minicpm4_config* cfg, int in_channels, int max_rows, vx_dit** out);
void vx_dit_destroy(vx_dit* dit);
/* in_proj [H, C], cond_proj [H, C], out_proj [C, H] (bf16, with f32 biases), and the two
 * TimestepEmbedding MLPs time_mlp / delta_time_mlp: linear_1 [H, H] + b, linear_2 [H, H] + b
 * (local_dit.rs:35-55). */
int vx_dit_load(vx_dit* dit, const uint16_t* in_w, const float* in_b, const uint16_t* cond_w, const float* cond_b,
                const uint16_t* out_w, const float* out_b, const uint16_t* t1_w, const float* t1_b,
                const uint16_t* t2_w, const float* t2_b, const uint16_t* dt1_w, const float* dt1_b,
                const uint16_t* dt2_w, const float* dt2_b);
/* Profiling: with VX_DIT_TRACE=1 set when the DiT first runs, the persistent decoder forward
 * records %globaltimer on every CTA of its last launch at each of its phases (8 per layer + 1):
 * [phase][CTA][4] = phase start, first segment's MMAs done (GEMM phases), CTA's work done, 0.
 * Copies phases * grid * 4 values into out (n entries at least). */
int vx_dit_trace(vx_dit* dit, unsigned long long* out, int n, int* grid, int* phases);
/* The same timeline for the batched greedy step's persistent decoder layers (VX_LM_BATCH_TRACE=1
 * set when the LM is created; the last batched step). */
int vx_lm_batch_trace(vx_lm* lm, unsigned long long* out, int n, int* grid, int* phases);
/* Decoder layer / final norm weights (as vx_lm_load_layer / vx_lm_load_norm). */
int vx_dit_load_layer(vx_dit* dit, int layer, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                      const uint16_t* o, const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                      const float* ln_in, const float* ln_post);
int vx_dit_load_norm(vx_dit* dit, const float* w);
/* VoxCpmLocDiTV2::forward (local_dit.rs:102-112): x [N, C, T], mu [N, C_mu], cond [N, C, Tc]
 * device; t and dt [N] host or device; out [N, C, T] device.  Synchronises. */
int vx_dit_forward(vx_dit* dit, const float* x, const float* mu, const float* t, const float* cond, const float* dt,
                   int N, int C_mu, int T, int Tc, float* out);
/* UnifiedCfm::forward + solve_euler (locdit/unified_cfm.rs:34-163), non-mean mode, with the
 * initial noise z [B, C, T] supplied by the caller (already scaled by temperature; the
 * reference draws it from the backend RNG, or zeros under VOXCPM_Z_ZERO).  mu [B, C_mu],
 * cond [B, C, Tc], x_out [B, C, T], all device.  Runs 2B DiT rows per step (cond | uncond
 * with mu zeroed), the fused CFG(-zero-star) + Euler update, and skips the DiT on the first
 * max(1, floor(0.04*(n+1))) steps when zero-star is on.  Polls vx_cancel between steps.
 * Synchronises. */
int vx_cfm_solve(vx_dit* dit, const float* mu, const float* cond, const float* z, int B, int C_mu, int T, int Tc,
                 int n_timesteps, float cfg_value, float sway_sampling_coef, int use_cfg_zero_star, float* x_out);

/* ----------------------------------------------------------------- AudioVAE decoder */

/* AudioVaeConfig (config.rs:219-309), decoder side.  Block i maps decoder_dim>>i to
 * decoder_dim>>(i+1) channels with stride rates[i]; every output channel count must be a
 * multiple of 64.  The sample-rate bucket is chosen once from out_sample_rate (sr_bucket,
 * audiovae/layers.rs:225-228); n_sr_boundaries = 0 disables SR conditioning. */
typedef struct {
  int latent_dim;
  int decoder_dim;
  const int* rates;
  int n_rates;
  int depthwise;       /* only 1 is supported (the shipped VoxCPM2 decoder) */
  int use_noise_block; /* only 0 is supported (NoiseBlock is off in VoxCPM2) */
  int out_sample_rate;
  const int* sr_boundaries;
  int n_sr_boundaries;
} vx_vae_config;

/* One CausalDecoderBlock (audiovae/decoder.rs:11-56) in checkpoint layouts: snake alpha [C_in];
 * ConvTranspose1d weight [C_in, C_out, 2*stride] bf16 + bias [C_out]; three
 * CausalResidualUnits (dilations 1, 3, 9): snake alphas [C_out], depthwise conv [C_out, 1, 7]
 * bf16 + bias, pointwise conv [C_out, C_out, 1] bf16 + bias; SampleRateConditionLayer
 * embedding tables [n_buckets, C_in] (scale, bias). */
typedef struct {
  const float* alpha;
  const uint16_t* up_w;
  const float* up_b;
  const float* res_alpha1[3];
  const uint16_t* res_w1[3];
  const float* res_b1[3];
  const float* res_alpha2[3];
  const uint16_t* res_w2[3];
  const float* res_b2[3];
  const float* sr_scale;
  const float* sr_bias;
} vx_vae_block_weights;

/* CausalDecoder::new (audiovae/decoder.rs:103-147). */
int vx_vae_create(vx_ctx* ctx, const vx_vae_config* cfg, vx_vae** out);
void vx_vae_destroy(vx_vae* vae);
/* DecoderFirstConv (decoder.rs:60-90), depthwise mode: dw [latent, 1, 7] + b, pw [dim, latent, 1] + b. */
int vx_vae_load_first(vx_vae* vae, const uint16_t* dw_w, const float* dw_b, const uint16_t* pw_w, const float* pw_b);
int vx_vae_load_block(vx_vae* vae, int block, const vx_vae_block_weights* w);
/* snake_out alpha [C_last] and the last CausalConv1d [1, C_last, 7] + bias [1] (decoder.rs:124-125). */
int vx_vae_load_out(vx_vae* vae, const float* alpha_out, const uint16_t* last_w, const float* last_b);
/* AudioVae::decode (audiovae/vae.rs:55-59): z [B, latent, T] -> wav [B, 1, T * prod(rates)],
 * device pointers.  Synchronises. */
int vx_vae_decode(vx_vae* vae, const float* z, int B, int T, float* wav);

/* Stateful chunked decode for B utterances, the counterpart of generate_stream's per-chunk
 * decode (voxcpm2/wrapper.rs:669-724), which re-decodes the whole accumulated latent every
 * chunk: here every causal layer keeps the tail of its input (the first depthwise conv's
 * last 6 latent frames, each transposed conv's last input frame, each residual unit's last
 * 6 x dilation inputs, the last conv's last 6), so vx_vae_stream_decode of a chunk of T new
 * latent frames costs T frames of work and writes exactly the T * prod(rates) samples that
 * decoding the whole latent would give for them (bit for bit).  Needs the tcgen05 convs
 * (latent a multiple of 64).  vx_vae_stream_reset starts a new utterance.  z [B, latent, T]
 * and wav [B, 1, T * prod(rates)] are device pointers; the call synchronises.  One stream per
 * VAE at a time: decodes share the VAE's work buffers. */
int vx_vae_stream_create(vx_vae* vae, int B, vx_vae_stream** out);
void vx_vae_stream_destroy(vx_vae_stream* s);
int vx_vae_stream_reset(vx_vae_stream* s);
int vx_vae_stream_decode(vx_vae_stream* s, const float* z, int T, float* wav);

/* ----------------------------------------------------------------- synthesis */

/* GenerateOptions (voxcpm2/wrapper.rs:146-187) as this library's synthesis loop uses them. */
typedef struct {
  float cfg_value;          /* classifier-free guidance scale (default 2.0) */
  int inference_timesteps;  /* Euler steps of the CFM solve (default 10) */
  int max_len;              /* latent patches to generate (the loop has no stop head) */
  int patch_size;           /* frames per patch (VoxCPM2: 4) */
  float sway_sampling_coef; /* dit_step passes 1.0 (voxcpm2/model.rs:236) */
  int use_cfg_zero_star;    /* dit_step passes true (voxcpm2/model.rs:237) */
} vx_generate_options;

/* One utterance end to end, shaped like VoxCpm2Model::inference + VoxCPM::generate
 * (voxcpm2/model.rs:301-375, wrapper.rs:401-423): greedy decode of the prompt ids with the
 * LM (graph-replayed steps); after decode step i, a CFM solve with mu = the LM's final-norm
 * hidden, cond = the previous patch (zeros first) and z = noise[i] ([C, P]; noise holds
 * max_len patches, host or device); patches stacked [C, max_len*P] (stack_pred_feats,
 * model.rs:283-287) and decoded by the VAE.  wav_out (host or device) receives
 * max_len*P*prod(rates) samples; latent_out (optional) the stacked latent.  The three
 * objects must share one context.  vx_cancel is polled every step (model.rs:330-334). */
int vx_generate(vx_lm* lm, vx_dit* dit, vx_vae* vae, const int32_t* prompt_ids, int n_prompt,
                const vx_generate_options* opts, const float* noise, float* wav_out, float* latent_out);

/* vx_generate for B utterances at once: the LM decodes the B prompts (equal lengths,
 * prompt_ids [B][n_prompt]) as B rows of one batched step (few-row GEMMs) and each patch's CFM
 * solve runs the B latents together; no reference counterpart beyond running B generate calls
 * (the reference is one utterance per VoxCPM).  noise [B][max_len][C][P]; wav_out
 * [B][max_len*P*prod(rates)]; latent_out (optional) [B][C][max_len*P].  Needs the LM created
 * with max_batch >= B and the DiT with max_rows >= 2B. */
int vx_generate_batch(vx_lm* lm, vx_dit* dit, vx_vae* vae, const int32_t* prompt_ids, int B, int n_prompt,
                      const vx_generate_options* opts, const float* noise, float* wav_out, float* latent_out);

/* ----------------------------------------------------------------- VoxCPM2 model */

/* VoxCpm2Model (voxcpm2/model.rs:22-37) over model objects created on one context: the base
 * LM (MiniCpmModel with its tied vocabulary, max_batch 1), the residual LM (vocab_size 0,
 * VoxCpm2Config::residual_lm_config, config.rs:421-427), the local encoder's MiniCPM-4
 * (vocab_size 0, encoder_lm_config, config.rs:430-440) and the LocDiT (dit_lm_config).  The
 * model keeps pointers to them; destroy it before them.  feat_dim D and patch_size P
 * (config.rs:318-321), scalar-quantization latent / scale (config.rs:326-329); max_len caps
 * the AR steps of one inference call. */
typedef struct vx_voxcpm2 vx_voxcpm2;

/* The projection weights of VoxCpm2Model::new (model.rs:41-100), bf16 [out, in] bit
 * patterns and f32 vectors (host or device pointers). */
typedef struct {
  const float* special_token;   /* VoxCpmLocEnc.special_token [enc_hidden] (locenc.rs:11) */
  const uint16_t* enc_in_w;     /* VoxCpmLocEnc.in_proj [enc_hidden, D] */
  const float* enc_in_b;
  const uint16_t* enc_to_lm_w;  /* [lm_hidden, enc_hidden] */
  const float* enc_to_lm_b;
  const uint16_t* lm_to_dit_w;  /* [dit_hidden, lm_hidden] */
  const float* lm_to_dit_b;
  const uint16_t* res_to_dit_w; /* [dit_hidden, lm_hidden] */
  const float* res_to_dit_b;
  const uint16_t* fusion_w;     /* fusion_concat_proj [lm_hidden, 2 * lm_hidden] */
  const float* fusion_b;
  const uint16_t* stop_proj_w;  /* [lm_hidden, lm_hidden] */
  const float* stop_proj_b;
  const uint16_t* stop_head_w;  /* [2, lm_hidden], no bias */
  const uint16_t* fsq_in_w;     /* ScalarQuantizationLayer.in_proj [latent, lm_hidden] (fsq.rs:17) */
  const float* fsq_in_b;
  const uint16_t* fsq_out_w;    /* ScalarQuantizationLayer.out_proj [lm_hidden, latent] */
  const float* fsq_out_b;
} vx_voxcpm2_weights;

int vx_voxcpm2_create(vx_lm* base_lm, vx_lm* residual_lm, vx_lm* encoder, vx_dit* dit, int feat_dim, int patch_size,
                      int sq_latent_dim, int sq_scale, int max_len, vx_voxcpm2** out);
void vx_voxcpm2_destroy(vx_voxcpm2* m);
int vx_voxcpm2_load(vx_voxcpm2* m, const vx_voxcpm2_weights* w);
/* VoxCpmLocEnc::forward (locenc.rs:32-44) for N patches: feat [N, P, D] (device) -> the cls
 * rows out [N, enc_hidden] (device).  Synchronises. */
int vx_locenc_forward(vx_voxcpm2* m, const float* feat, int N, float* out);
/* VoxCpm2Model::inference (model.rs:301-375) for one sequence: prefill (model.rs:128-207)
 * over text_token [S] ids, text_mask / feat_mask [S] (0 or 1) and feat [S, P, D], then
 * dit_step / lm_step (model.rs:215-279) until the stop head fires at a step i > min_len or
 * max_len patches exist.  noise [max_len, D, P] is each step's CFM noise z (the reference
 * draws it from the backend RNG, unified_cfm.rs:47-52); the CFM runs with sway 1 and
 * CFG-zero-star as dit_step passes them.  latent_out receives [D, n * P] (stack_pred_feats,
 * model.rs:283-287) with n written to *n_patches; stop_logits_out (optional) [n, 2].  The
 * stop flag stays on the device: the host reads step i's flag after queueing step i + 1.
 * vx_cancel is polled every step (model.rs:323-328).  Inputs may be host or device memory. */
int vx_voxcpm2_inference(vx_voxcpm2* m, const int32_t* text_token, const float* text_mask, const float* feat,
                         const float* feat_mask, int S, int min_len, int max_len, int inference_timesteps,
                         float cfg_value, const float* noise, float* latent_out, int* n_patches,
                         float* stop_logits_out);
/* The inference loop in steps, for streaming (VoxCPM::generate_stream, wrapper.rs:456-492,
 * 680-724): vx_voxcpm2_begin runs the prefill with the same arguments as
 * vx_voxcpm2_inference; each vx_voxcpm2_advance runs up to max_patches more AR steps and
 * writes the new patches' latent [D, n_new * P] (host or device) to latent_out; *finished
 * becomes 1 once the stop head fired at a step i > min_len or max_len patches exist.  The
 * concatenated latents equal vx_voxcpm2_inference's. */
int vx_voxcpm2_begin(vx_voxcpm2* m, const int32_t* text_token, const float* text_mask, const float* feat,
                     const float* feat_mask, int S, int min_len, int max_len, int inference_timesteps,
                     float cfg_value, const float* noise);
int vx_voxcpm2_advance(vx_voxcpm2* m, int max_patches, float* latent_out, int* n_new, int* finished);
/* VoxCPM::generate (wrapper.rs:401-423) without the tokenizer: vx_voxcpm2_inference, then
 * decode_latent_to_samples (wrapper.rs:616-629) through the VAE.  wav_out (host or device)
 * must hold max_len * P * prod(rates) samples; *n_samples receives the count written. */
int vx_voxcpm2_generate(vx_voxcpm2* m, vx_vae* vae, const int32_t* text_token, const float* text_mask,
                        const float* feat, const float* feat_mask, int S, int min_len, int max_len,
                        int inference_timesteps, float cfg_value, const float* noise, float* wav_out,
                        int* n_samples);

/* ----------------------------------------------------------------- checkpoints */

/* Element types of checkpoint tensors (safetensors dtypes / torch storage types). */
enum { VX_DT_F32 = 0, VX_DT_F16 = 1, VX_DT_BF16 = 2, VX_DT_F64 = 3, VX_DT_I64 = 4, VX_DT_I32 = 5, VX_DT_I16 = 6,
       VX_DT_I8 = 7, VX_DT_U8 = 8, VX_DT_BOOL = 9 };

/* A checkpoint file opened on the host (load_single / load_single_pth, weights.rs:264-367):
 * a .safetensors file, or a PyTorch zip checkpoint (.pth / .pt, torch.save) whose nested
 * dicts are flattened with '.' and whose "state_dict." / "model_state_dict." / "module."
 * prefixes are stripped (strip_pth_top_level, weights.rs:400-411).  The file is
 * memory-mapped until vx_weights_close.  Errors are reported by vx_weights_last_error
 * (this thread's last failure). */
typedef struct vx_weights vx_weights;
int vx_weights_open(const char* path, vx_weights** out);
void vx_weights_close(vx_weights* w);
const char* vx_weights_last_error(void);
int vx_weights_count(const vx_weights* w);
const char* vx_weights_name(const vx_weights* w, int i);
int vx_weights_find(const vx_weights* w, const char* name);
/* dtype and shape of tensor i; returns its rank (-1 if i is out of range). */
int vx_weights_info(const vx_weights* w, int i, int* dtype, int64_t* shape, int max_dims);
/* Tensor `name` converted to out_dtype (VX_DT_F32, or VX_DT_BF16 rounded to nearest even)
 * into host memory of n_elems elements.  A "<stem>.weight" that the file stores as a
 * weight_norm pair (<stem>.weight_g, <stem>.weight_v) is materialised:
 * w[o, ...] = g[o] * v[o, ...] / max(||v[o, :]||, 1e-12) (materialize_weight_norm,
 * weights.rs:447-471). */
int vx_weights_read(const vx_weights* w, const char* name, int out_dtype, void* out, size_t n_elems);

/* Model loaders over the upstream checkpoint key layout (the reference's module paths,
 * weights.rs:56-133): <prefix>layers.<i>.self_attn.{q,k,v,o}_proj.weight (or a fused
 * qkv_proj), mlp.{gate,up,down}_proj.weight (or gate_up_proj), input_layernorm /
 * post_attention_layernorm, <prefix>norm.weight, <prefix>embed_tokens.weight (with a
 * vocabulary).  Shapes are checked against the model (VX_ERR_SHAPE). */
int vx_lm_load_weights(vx_lm* lm, const vx_weights* w, const char* prefix);
/* VoxCpmLocDiTV2 (local_dit.rs:58-67): <prefix>{in,cond,out}_proj, time_mlp / delta_time_mlp
 * .linear_{1,2}, decoder.*  (VoxCPM2: prefix "feat_decoder.estimator."). */
int vx_dit_load_weights(vx_dit* dit, const vx_weights* w, const char* prefix);
/* AudioVAE decoder from the checkpoint's nn.Sequential keys (remap_audiovae_key,
 * weights.rs:140-262) under <prefix>decoder.: model.0 / model.1 (first depthwise / pointwise
 * conv), model.<2+i>.block.{0: snake, 1: transposed conv, 2-4: residual units with block.0-3
 * = snake1, conv1, snake2, conv2}, model.<2+n> snake_out, model.<3+n> last conv,
 * sr_cond_model.<2+i>.{scale,bias}_embed.weight; weight_norm pairs are materialised. */
int vx_vae_load_weights(vx_vae* vae, const vx_weights* w, const char* prefix);
/* The whole VoxCpm2Model (model.rs:22-37) from model.safetensors / model.pth: base_lm.,
 * residual_lm., feat_encoder.{special_token, in_proj, encoder.}, feat_decoder.estimator.,
 * fsq_layer.{in,out}_proj, enc_to_lm_proj, lm_to_dit_proj, res_to_dit_proj,
 * fusion_concat_proj, stop_proj, stop_head. */
int vx_voxcpm2_load_weights(vx_voxcpm2* m, const vx_weights* w);

#ifdef __cplusplus
}
#endif

#endif /* VOXCPM_B200_H */
