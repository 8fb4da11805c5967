// MiniCPM-4 model object: weights, static KV cache, prefill, the batch-1 decode step and
// the graph-captured greedy decode loop (reference src/minicpm4/model.rs, layer.rs,
// attention.rs, mlp.rs, cache.rs).
//
// HBM layout (per model):
//   weights  bf16, per layer: wqkv [(nh+2nkv)*d, H] | wo [H, nh*d] | wgu [2I, H] | wd [H, I]
//            (checkpoint [out, in] layout, q|k|v and gate|up fused along out)
//   norms    f32 [H] (ln_in, ln_post per layer; final norm)
//   embed    bf16 [V, H] (tied: input embedding and greedy LM head)
//   KV cache f32 [L][B][nkv][max_length][d] for K and for V (post-RoPE K)
//   state    device ints: position of the token being decoded, greedy step index, token ids
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "dit_persist.cuh"
#include "persist.cuh"
#include "runtime.cuh"

using namespace vx;

namespace {

struct LmLayer {
  uint16_t* wqkv = nullptr;
  uint16_t* wo = nullptr;
  uint16_t* wgu = nullptr;
  uint16_t* wd = nullptr;
  float* ln_in = nullptr;
  float* ln_post = nullptr;
};

}  // namespace

struct vx_lm {
  vx_ctx* ctx = nullptr;
  vx_minicpm4_config cfg{};
  int H = 0, I = 0, nh = 0, nkv = 0, d = 0, L = 0, V = 0, qs = 0, ks = 0;
  float res_scale = 1.f, emb_scale = 1.f, attn_scale = 1.f;
  int max_batch = 1, max_length = 0;
  int cur_len = 0;  // StaticKvCache::current_length (host mirror)

  std::vector<LmLayer> layers;
  void* weight_slab = nullptr;
  float* norm_w = nullptr;
  uint16_t* embed = nullptr;
  RopeParams* rope = nullptr;  // device, nullptr when no_rope
  float* rope_tab = nullptr;   // cos / sin of positions 0..ATT_FUSED_ROPE_MAX_S-1 [pos][2][d/2]
  float* kcache = nullptr;
  float* vcache = nullptr;

  // device state for the graph-replayed decode step
  int* d_pos = nullptr;
  int* d_step = nullptr;
  int* d_tokens = nullptr;
  // batch-1 decode buffers
  float* x = nullptr;       // residual stream [H]
  float* q = nullptr;       // [nh*d]
  float* attn = nullptr;    // [nh*d]
  float* act = nullptr;     // [I]
  float* logits = nullptr;  // [V]
  float* hid_norm = nullptr;  // final-norm hidden of the last greedy pick [H]
  float* attn_partials = nullptr;
  unsigned* attn_counters = nullptr;
  float2* argmax_partials = nullptr;
  unsigned* argmax_counter = nullptr;
  int attn_nsplit = 16;
  // prefill buffers (grown on demand)
  size_t pf_rows = 0;
  float *pf_x = nullptr, *pf_xn = nullptr, *pf_qkv = nullptr, *pf_q = nullptr, *pf_attn = nullptr,
        *pf_gu = nullptr, *pf_act = nullptr, *pf_k = nullptr, *pf_v = nullptr;
  int* pf_ids = nullptr;
  int pf_ids_cap = 0;

  // batched greedy decode: B rows in lockstep (equal prompt lengths), one shared position
  int bt_B = 0;                         // rows of the captured batch step graph
  cudaGraphExec_t bstep_exec = nullptr;
  unsigned long long bstep_kernels = 0;
  float *bx = nullptr, *bxn = nullptr, *bqkv = nullptr, *bq = nullptr, *battn = nullptr, *bgu = nullptr,
        *bact = nullptr, *blogits = nullptr, *bhid = nullptr;
  int* btokens = nullptr;  // [max_length + 8][max_batch]
  // the batched step's decoder layers as one persistent launch (dit_persist.cu, decode
  // attention); env VX_LM_BATCH_PERSIST=0: the per-kernel layers
  PersistStack bp;
  bool bp_on = true;
  bool bt_persist = false;  // the captured batch step uses it
  cudaGraphExec_t step_exec = nullptr;
  unsigned long long step_kernels = 0;
  // persistent decode step (one launch per token), when the shape allows it
  int pk_grid = 0;
  float* x_mid = nullptr;              // residual stream after attention [H]
  PersistLayer* pk_layers = nullptr;   // device [L]
  unsigned* pk_cnt = nullptr;          // phase counters [5L + 2]
  float* pk_att_part = nullptr;        // attention split partials of the persistent step
  long long* pk_xacc = nullptr;        // its fixed-point residual accumulators [2][H]
  uint16_t* pk_wdt = nullptr;          // its transposed down_proj weights [L][I][H]
  LinearWorkspace ws;  // tcgen05 few-row GEMM workspace (prefill, non-causal forward)
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  float t_prefill_ms = 0.f, t_decode_ms = 0.f;
  int pos_host = 0;

  size_t kv_layer_stride() const { return (size_t)max_batch * nkv * max_length * d; }
  float* kc(int l, int b) { return kcache + l * kv_layer_stride() + (size_t)b * nkv * max_length * d; }
  float* vc(int l, int b) { return vcache + l * kv_layer_stride() + (size_t)b * nkv * max_length * d; }
};

namespace {

void free_prefill(vx_lm* lm) {
  for (float** p : {&lm->pf_x, &lm->pf_xn, &lm->pf_qkv, &lm->pf_q, &lm->pf_attn, &lm->pf_gu, &lm->pf_act,
                    &lm->pf_k, &lm->pf_v}) {
    if (*p) cudaFree(*p);
    *p = nullptr;
  }
  lm->pf_rows = 0;
}

int ensure_prefill(vx_lm* lm, size_t rows, int B, int S, bool need_kv) {
  if (rows <= lm->pf_rows && (!need_kv || lm->pf_k)) return VX_OK;
  free_prefill(lm);
  const size_t H = lm->H, q = lm->qs, qkv = lm->qs + 2 * lm->ks, I = lm->I;
  bool ok = cudaMalloc(&lm->pf_x, rows * H * 4) == cudaSuccess && cudaMalloc(&lm->pf_xn, rows * H * 4) == cudaSuccess &&
            cudaMalloc(&lm->pf_qkv, rows * qkv * 4) == cudaSuccess && cudaMalloc(&lm->pf_q, rows * q * 4) == cudaSuccess &&
            cudaMalloc(&lm->pf_attn, rows * q * 4) == cudaSuccess && cudaMalloc(&lm->pf_gu, rows * 2 * I * 4) == cudaSuccess &&
            cudaMalloc(&lm->pf_act, rows * I * 4) == cudaSuccess &&
            cudaMalloc(&lm->pf_k, rows * lm->ks * 4) == cudaSuccess && cudaMalloc(&lm->pf_v, rows * lm->ks * 4) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    free_prefill(lm);
    return fail(lm->ctx, VX_ERR_OOM, "prefill buffers (%zu rows) allocation failed", rows);
  }
  lm->pf_rows = rows;
  return VX_OK;
}

// ----------------------------------------------------------------- kernel sequences

// One decoder layer for batch row 0 at the device position *d_pos (or `pos` when
// pos_from_device is false): 5 launches.
int enqueue_layer_step(vx_lm* lm, int l, cudaStream_t st, bool pos_from_device, int pos,
                       cudaEvent_t* ev_after = nullptr) {
  vx_ctx* ctx = lm->ctx;
  int evi = 0;
  auto mark = [&]() -> cudaError_t { return ev_after ? cudaEventRecord(ev_after[evi++], st) : cudaSuccess; };
  const LmLayer& w = lm->layers[l];
  const bool pdl = ctx->pdl;
  // (1) input_layernorm -> qkv_proj -> LongRoPE -> KV cache write  (layer.rs:64-66, attention.rs:102-127)
  GemvArgs a = {};
  a.W = w.wqkv;
  a.N = lm->qs + 2 * lm->ks;
  a.K = lm->H;
  a.x = lm->x;
  a.norm_w = w.ln_in;
  a.eps = lm->cfg.rms_norm_eps;
  a.map_mode = MAP_ROPE_PAIRS;
  a.map_param = lm->d / 16;
  a.groups_per_cta = 2 * pick_groups(a.N / 16, ctx->gemv_ctas);
  a.nh = lm->nh;
  a.nkv = lm->nkv;
  a.hd = lm->d;
  a.rope = lm->rope;
  a.pos_ptr = pos_from_device ? lm->d_pos : nullptr;
  a.pos_val = pos;
  a.q_out = lm->q;
  a.kcache = lm->kc(l, 0);
  a.vcache = lm->vc(l, 0);
  a.s_max = lm->max_length;
  // L2 prefetch chain: every weight-streaming kernel prefetches the next one's weights
  const bool pf = ctx->l2_prefetch;
  const size_t H = lm->H, I = lm->I;
  if (pf) {
    a.pf_ptr = w.wo;
    a.pf_bytes = H * lm->qs * 2;
  }
  VX_CUDA(ctx, launch_gemv(a, EPI_QKV_ROPE, st, pdl, ctx->dev_err));
  VX_CUDA(ctx, mark());
  // (2) sdpa over the cached prefix 0..pos+1 (attention.rs:129-150)
  AttnDecodeArgs ad = {lm->q, lm->kc(l, 0), lm->vc(l, 0), 1, lm->nh, lm->nkv, lm->d, lm->max_length,
                       pos_from_device ? lm->d_pos : nullptr, pos + 1, lm->attn_scale, lm->attn_nsplit,
                       lm->attn_partials, lm->attn_counters, lm->attn};
  VX_CUDA(ctx, launch_attn_decode(ad, st, pdl));
  VX_CUDA(ctx, mark());
  // (3) o_proj + residual (attention.rs:153, layer.rs:67)
  GemvArgs o = {};
  o.W = w.wo;
  o.N = lm->H;
  o.K = lm->qs;
  o.x = lm->attn;
  o.y = lm->x;
  o.residual = lm->x;
  o.res_scale = lm->res_scale;
  o.groups_per_cta = pick_groups(o.N / 8, ctx->gemv_ctas);
  if (pf) {
    o.pf_ptr = w.wgu;
    o.pf_bytes = 2 * I * H * 2;
  }
  VX_CUDA(ctx, launch_gemv(o, EPI_STORE, st, pdl, ctx->dev_err));
  VX_CUDA(ctx, mark());
  // (4) post_attention_layernorm -> gate_up -> silu(gate)*up (layer.rs:69-71, mlp.rs:29-33)
  GemvArgs g = {};
  g.W = w.wgu;
  g.N = 2 * lm->I;
  g.K = lm->H;
  g.x = lm->x;
  g.norm_w = w.ln_post;
  g.eps = lm->cfg.rms_norm_eps;
  g.map_mode = MAP_GATE_UP;
  g.map_param = lm->I / 8;
  g.groups_per_cta = 2 * pick_groups(lm->I / 8, ctx->gemv_ctas);
  g.inter = lm->I;
  g.act = lm->act;
  if (pf) {
    g.pf_ptr = w.wd;
    g.pf_bytes = H * I * 2;
  }
  VX_CUDA(ctx, launch_gemv(g, EPI_SILU_MUL, st, pdl, ctx->dev_err));
  VX_CUDA(ctx, mark());
  // (5) down_proj + residual (mlp.rs:33, layer.rs:72)
  GemvArgs dn = {};
  dn.W = w.wd;
  dn.N = lm->H;
  dn.K = lm->I;
  dn.x = lm->act;
  dn.y = lm->x;
  dn.residual = lm->x;
  dn.res_scale = lm->res_scale;
  dn.groups_per_cta = pick_groups(dn.N / 8, ctx->gemv_ctas);
  if (pf && l + 1 < lm->L) {
    dn.pf_ptr = lm->layers[l + 1].wqkv;
    dn.pf_bytes = (size_t)(lm->qs + 2 * lm->ks) * H * 2;
  } else if (pf && lm->embed) {
    dn.pf_ptr = lm->embed;  // the head of the greedy LM head's table
    dn.pf_bytes = std::min<size_t>((size_t)lm->V * H * 2, 48u << 20);
  }
  VX_CUDA(ctx, launch_gemv(dn, EPI_STORE, st, pdl, ctx->dev_err));
  VX_CUDA(ctx, mark());
  return VX_OK;
}

// Greedy LM head over the tied embedding: final norm -> logits -> argmax -> next input.
int enqueue_lm_head(vx_lm* lm, cudaStream_t st, bool advance_pos, bool write_logits) {
  GemvArgs h = {};
  h.W = lm->embed;
  h.N = lm->V;
  h.K = lm->H;
  h.x = lm->x;
  h.norm_w = lm->norm_w;
  h.eps = lm->cfg.rms_norm_eps;
  h.groups_per_cta = pick_groups(lm->V / 8, lm->ctx->gemv_ctas);
  h.logits = write_logits ? lm->logits : nullptr;
  h.partials = lm->argmax_partials;
  h.counter = lm->argmax_counter;
  h.token_out = lm->d_tokens;
  h.step_ptr = lm->d_step;
  h.embed = lm->embed;
  h.embed_dim = lm->H;
  h.embed_scale = lm->emb_scale;
  h.next_x = lm->x;
  h.pos_inc = advance_pos ? lm->d_pos : nullptr;
  h.norm_out = lm->hid_norm;
  VX_CUDA(lm->ctx, launch_gemv(h, EPI_ARGMAX, st, lm->ctx->pdl, lm->ctx->dev_err));
  return VX_OK;
}

int enqueue_decode_step(vx_lm* lm, cudaStream_t st) {
  for (int l = 0; l < lm->L; ++l) {
    int rc = enqueue_layer_step(lm, l, st, true, 0);
    if (rc) return rc;
  }
  return enqueue_lm_head(lm, st, true, true);
}

// The whole decode step as one persistent launch (batch row 0).
cudaError_t enqueue_persist_step(vx_lm* lm, cudaStream_t st, bool cooperative,
                                 unsigned long long* trace = nullptr) {
  PersistArgs a = {};
  a.L = lm->L;
  a.H = lm->H;
  a.I = lm->I;
  a.nh = lm->nh;
  a.nkv = lm->nkv;
  a.d = lm->d;
  a.V = lm->V;
  a.s_max = lm->max_length;
  a.eps = lm->cfg.rms_norm_eps;
  a.res_scale = lm->res_scale;
  a.attn_scale = lm->attn_scale;
  a.emb_scale = lm->emb_scale;
  a.layers = lm->pk_layers;
  a.final_norm = lm->norm_w;
  a.embed = lm->embed;
  a.rope = lm->rope;
  a.kcache = lm->kc(0, 0);
  a.vcache = lm->vc(0, 0);
  a.kv_layer_stride = lm->kv_layer_stride();
  a.pos = lm->d_pos;
  a.step = lm->d_step;
  a.tokens = lm->d_tokens;
  a.x0 = lm->x;
  a.xacc = lm->pk_xacc;
  a.x1 = lm->x_mid;
  a.q = lm->q;
  a.logits = lm->logits;
  a.hid_norm = lm->hid_norm;
  a.att_part = lm->pk_att_part;
  a.am_part = lm->argmax_partials;
  a.phase_cnt = lm->pk_cnt;
  a.err = lm->ctx->dev_err;
  a.trace = trace;
  a.pf_stages = lm->ctx->persist_pf;
  a.evict_first = lm->ctx->persist_ef;
  a.inflight = lm->ctx->persist_inflight;
  a.mlp_pf = lm->ctx->persist_mlp_pf;
  a.merge_tiles = lm->ctx->persist_merge_tiles;
  return launch_persist(a, lm->pk_grid, lm->ctx->persist_nst, st, cooperative);
}

int capture_step(vx_lm* lm, int mode, cudaGraphExec_t* exec) {
  // mode 0: per-kernel step; 1: persistent, cooperative launch
  vx_ctx* ctx = lm->ctx;
  cudaGraph_t graph = nullptr;
  const unsigned long long before = g_launches;
  cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaStreamBeginCapture");
  int rc = VX_OK;
  cudaError_t le = cudaSuccess;
  if (mode == 0)
    rc = enqueue_decode_step(lm, ctx->stream);
  else
    le = enqueue_persist_step(lm, ctx->stream, mode == 1);
  e = cudaStreamEndCapture(ctx->stream, &graph);
  lm->step_kernels = g_launches - before;  // captured, not launched
  g_launches = before;
  if (rc || le != cudaSuccess || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    if (rc) return rc;
    return cuda_fail(ctx, le != cudaSuccess ? le : e, "decode step capture");
  }
  e = cudaGraphInstantiate(exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(ctx, e, "cudaGraphInstantiate");
  }
  return VX_OK;
}

int build_step_graph(vx_lm* lm) {
  if (lm->step_exec) return VX_OK;
  if (lm->pk_grid > 0) {
    // The persistent step's CTAs wait on one another, so it needs a cooperative launch (every
    // CTA resident at once).  If that cannot be captured, use the per-kernel step: a plain
    // launch could leave CTAs unscheduled behind other work and end in VX_ERR_TIMEOUT.
    if (capture_step(lm, 1, &lm->step_exec) == VX_OK) return VX_OK;
    cudaGetLastError();
    lm->pk_grid = 0;
  }
  return capture_step(lm, 0, &lm->step_exec);
}

// ----------------------------------------------------------------- batched decode step

int ensure_batch(vx_lm* lm) {
  if (lm->bx) return VX_OK;
  const size_t Bm = lm->max_batch, H = lm->H, I = lm->I, qkvw = lm->qs + 2 * lm->ks;
  bool ok = cudaMalloc(&lm->bx, Bm * H * 4) == cudaSuccess && cudaMalloc(&lm->bxn, Bm * H * 4) == cudaSuccess &&
            cudaMalloc(&lm->bqkv, Bm * qkvw * 4) == cudaSuccess && cudaMalloc(&lm->bq, Bm * lm->qs * 4) == cudaSuccess &&
            cudaMalloc(&lm->battn, Bm * lm->qs * 4) == cudaSuccess && cudaMalloc(&lm->bgu, Bm * 2 * I * 4) == cudaSuccess &&
            cudaMalloc(&lm->bact, Bm * I * 4) == cudaSuccess &&
            cudaMalloc(&lm->blogits, Bm * (size_t)lm->V * 4) == cudaSuccess &&
            cudaMalloc(&lm->bhid, Bm * H * 4) == cudaSuccess &&
            cudaMalloc(&lm->btokens, (size_t)(lm->max_length + 8) * Bm * 4) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    return fail(lm->ctx, VX_ERR_OOM, "batched decode buffers allocation failed");
  }
  return VX_OK;
}

// Greedy head for B rows: final norm (kept as the hidden the DiT consumes), logits over the
// tied embedding, per-row argmax -> token and next input embedding, then step (and position).
int enqueue_batch_head(vx_lm* lm, int B, cudaStream_t st, bool advance_pos, bool normed = false) {
  vx_ctx* ctx = lm->ctx;
  const int H = lm->H;
  if (!normed)  // else bhid already holds the final-norm rows
    VX_CUDA(ctx, launch_rmsnorm_residual(lm->bx, nullptr, lm->norm_w, 1.f, lm->cfg.rms_norm_eps, B, H, nullptr,
                                         lm->bhid, st));
  int rc = linear(ctx, &lm->ws, lm->bhid, H, B, lm->V, H, lm->embed, nullptr, nullptr, 1.f, lm->blogits, lm->V, st);
  if (rc) return rc;
  VX_CUDA(ctx, launch_argmax_rows(lm->blogits, B, lm->V, lm->d_step, lm->btokens, lm->max_batch, lm->embed, H,
                                  lm->emb_scale, lm->bx, st));
  VX_CUDA(ctx, launch_advance(lm->d_pos, lm->d_step, advance_pos, st));
  return VX_OK;
}

// One decode step for B rows at the device position (forward_step, model.rs:64-84, per row):
// per layer RMSNorm -> qkv (few-row GEMM) -> LongRoPE + KV write -> split-K attention ->
// o_proj + residual -> RMSNorm -> gate|up -> SiLU*up -> down + residual; then the head.
int enqueue_batch_step(vx_lm* lm, int B, cudaStream_t st) {
  vx_ctx* ctx = lm->ctx;
  const int H = lm->H, I = lm->I, qkvw = lm->qs + 2 * lm->ks;
  const float eps = lm->cfg.rms_norm_eps;
  int rc = VX_OK;
  if (lm->bt_persist) {  // every layer and the final norm in one launch: bx -> bhid
    DitPersistArgs a = persist_stack_args(lm->bp, B, 1, lm->bx, lm->bhid, ctx->dev_err);
    a.att_mode = DP_ATT_DECODE;
    a.kcache = lm->kcache;
    a.vcache = lm->vcache;
    a.kv_layer_stride = lm->kv_layer_stride();
    a.max_len = lm->max_length;
    a.pos = lm->d_pos;
    // the o_proj units go to the CTAs without an attention unit (B nkv of them have one): their
    // weight tiles stream in while those walk the cache
    a.cta_off[DP_KIND_O] = std::min(B * lm->nkv, std::max(0, lm->bp.grid - a.ncta[DP_KIND_O]));
    VX_CUDA(ctx, launch_dit_persist(a, lm->bp.grid, st));
    return enqueue_batch_head(lm, B, st, true, true);
  }
  // the RMSNorm and SiLU*up kernels write the few-row GEMMs' split operand themselves
  uint16_t* xs = lm->ws.scratch ? tc_gemm_presplit_buffer(lm->ws.scratch) : nullptr;
  const bool ps_qkv = presplit_ok(ctx, &lm->ws, B, qkvw, H), ps_gu = presplit_ok(ctx, &lm->ws, B, 2 * I, H),
             ps_d = presplit_ok(ctx, &lm->ws, B, H, I);
  for (int l = 0; l < lm->L; ++l) {
    const LmLayer& w = lm->layers[l];
    VX_CUDA(ctx, launch_rmsnorm_residual(lm->bx, nullptr, w.ln_in, 1.f, eps, B, H, nullptr, ps_qkv ? nullptr : lm->bxn,
                                         st, ps_qkv ? xs : nullptr));
    rc = ps_qkv ? linear_presplit(ctx, &lm->ws, B, qkvw, H, w.wqkv, nullptr, nullptr, 1.f, lm->bqkv, qkvw, st)
                : linear(ctx, &lm->ws, lm->bxn, H, B, qkvw, H, w.wqkv, nullptr, nullptr, 1.f, lm->bqkv, qkvw, st);
    if (rc) return rc;
    VX_CUDA(ctx, launch_rope_scatter(lm->bqkv, B, 1, lm->nh, lm->nkv, lm->d, lm->rope, 0, lm->bq, lm->kc(l, 0),
                                     lm->vc(l, 0), lm->max_length, st, lm->d_pos));
    AttnDecodeArgs ad = {lm->bq, lm->kc(l, 0), lm->vc(l, 0), B, lm->nh, lm->nkv, lm->d, lm->max_length, lm->d_pos, 0,
                         lm->attn_scale, lm->attn_nsplit, lm->attn_partials, lm->attn_counters, lm->battn};
    VX_CUDA(ctx, launch_attn_decode(ad, st, false));
    if ((rc = linear(ctx, &lm->ws, lm->battn, lm->qs, B, H, lm->qs, w.wo, nullptr, lm->bx, lm->res_scale, lm->bx, H, st)))
      return rc;
    VX_CUDA(ctx, launch_rmsnorm_residual(lm->bx, nullptr, w.ln_post, 1.f, eps, B, H, nullptr, ps_gu ? nullptr : lm->bxn,
                                         st, ps_gu ? xs : nullptr));
    rc = ps_gu ? linear_presplit(ctx, &lm->ws, B, 2 * I, H, w.wgu, nullptr, nullptr, 1.f, lm->bgu, 2 * I, st)
               : linear(ctx, &lm->ws, lm->bxn, H, B, 2 * I, H, w.wgu, nullptr, nullptr, 1.f, lm->bgu, 2 * I, st);
    if (rc) return rc;
    VX_CUDA(ctx, launch_silu_mul(lm->bgu, B, I, lm->bact, st, ps_d ? xs : nullptr));
    rc = ps_d ? linear_presplit(ctx, &lm->ws, B, H, I, w.wd, nullptr, lm->bx, lm->res_scale, lm->bx, H, st)
              : linear(ctx, &lm->ws, lm->bact, I, B, H, I, w.wd, nullptr, lm->bx, lm->res_scale, lm->bx, H, st);
    if (rc) return rc;
  }
  return enqueue_batch_head(lm, B, st, true);
}

int build_batch_graph(vx_lm* lm, int B) {
  if (lm->bstep_exec && lm->bt_B == B) return VX_OK;
  vx_ctx* ctx = lm->ctx;
  if (lm->bstep_exec) {
    cudaGraphExecDestroy(lm->bstep_exec);
    lm->bstep_exec = nullptr;
  }
  // the persistent layers: buffers and maps before the capture
  lm->bt_persist = false;
  if (lm->bp_on && lm->bp.grid < 0) {
    LmStackView v;
    lm_stack_view(lm, &v);
    bool oom = false;
    persist_stack_prepare(lm->bp, v, lm->max_batch, getenv("VX_LM_BATCH_TRACE") != nullptr, &oom, lm->max_length);
    if (oom) return fail(ctx, VX_ERR_OOM, "persistent batch step: allocation or tensor maps failed");
  }
  if (lm->bp_on && lm->bp.grid > 0 && lm->bp.decode_ok && B <= lm->bp.rmax)
    lm->bt_persist = persist_stack_rows(lm->bp, (B + 31) / 32 * 32);
  cudaGraph_t graph = nullptr;
  const unsigned long long before = g_launches;
  VX_CUDA(ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_batch_step(lm, B, ctx->stream);
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
  lm->bstep_kernels = g_launches - before;  // captured, not launched
  g_launches = before;
  if (rc || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rc ? rc : cuda_fail(ctx, e, "batch decode step capture");
  }
  e = cudaGraphInstantiate(&lm->bstep_exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "cudaGraphInstantiate");
  lm->bt_B = B;
  return VX_OK;
}

int check_device_error(vx_ctx* ctx) { return vx_ctx_synchronize(ctx); }

}  // namespace

extern "C" {

int vx_lm_create(vx_ctx* ctx, const vx_minicpm4_config* cfg, int max_batch, int max_length, vx_lm** out) {
  if (!ctx || !cfg || !out) return VX_ERR_ARG;
  *out = nullptr;
  const int d = cfg->kv_channels > 0 ? cfg->kv_channels : cfg->hidden_size / cfg->num_attention_heads;
  if (cfg->hidden_size <= 0 || cfg->num_attention_heads <= 0 || cfg->num_key_value_heads <= 0 ||
      cfg->num_attention_heads % cfg->num_key_value_heads != 0 || cfg->num_hidden_layers < 0 ||
      cfg->intermediate_size <= 0 || max_batch <= 0 || max_length <= 0)
    return fail(ctx, VX_ERR_CONFIG, "lm_create: invalid config");
  if (cfg->hidden_size % 256 != 0 || cfg->intermediate_size % 256 != 0 || d % 16 != 0 ||
      (cfg->num_attention_heads * d) % 256 != 0)
    return fail(ctx, VX_ERR_CONFIG, "lm_create: hidden/intermediate/q widths must be multiples of 256, head_dim of 16");
  cudaSetDevice(ctx->device);
  vx_lm* lm = new vx_lm();
  lm->ctx = ctx;
  if (const char* e = getenv("VX_LM_BATCH_PERSIST")) lm->bp_on = atoi(e) != 0;
  lm->cfg = *cfg;
  lm->cfg.rope_short_factor = nullptr;
  lm->cfg.rope_long_factor = nullptr;
  lm->H = cfg->hidden_size;
  lm->I = cfg->intermediate_size;
  lm->nh = cfg->num_attention_heads;
  lm->nkv = cfg->num_key_value_heads;
  lm->d = d;
  lm->L = cfg->num_hidden_layers;
  lm->V = cfg->vocab_size;
  lm->qs = lm->nh * d;
  lm->ks = lm->nkv * d;
  lm->res_scale = (float)residual_scale_of(*cfg);
  lm->emb_scale = cfg->use_mup ? cfg->scale_emb : 1.0f;
  lm->attn_scale = (float)(1.0 / std::sqrt((double)d));  // MiniCpmAttention::new scale (attention.rs:48)
  lm->max_batch = max_batch;
  lm->max_length = max_length;
  lm->attn_nsplit = 32;  // upper bound; the kernel activates ceil(len/32) of them

  auto fail_free = [&](int code, const char* msg) {
    vx_lm_destroy(lm);
    return fail(ctx, code, "%s", msg);
  };
  if (!cfg->no_rope) {
    RopeParams rp;
    std::string err;
    int rc = fill_rope_params(*cfg, &rp, &err);
    if (rc) {
      delete lm;
      return fail(ctx, rc, "%s", err.c_str());
    }
    if (cudaMalloc(&lm->rope, sizeof(RopeParams)) != cudaSuccess ||
        cudaMemcpy(lm->rope, &rp, sizeof(RopeParams), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMalloc(&lm->rope_tab, (size_t)ATT_FUSED_ROPE_MAX_S * lm->d * 4) != cudaSuccess ||
        launch_rope_table(lm->rope, ATT_FUSED_ROPE_MAX_S, lm->d / 2, lm->rope_tab, 0) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess)
      return fail_free(VX_ERR_OOM, "rope params allocation failed");
  }
  const size_t H = lm->H, I = lm->I;
  const size_t per_layer = ((size_t)(lm->qs + 2 * lm->ks) * H + H * lm->qs + 2 * I * H + H * I) * 2 + 2 * H * 4;
  if (cudaMalloc(&lm->weight_slab, per_layer * std::max(1, lm->L) + 256) != cudaSuccess)
    return fail_free(VX_ERR_OOM, "weight allocation failed");
  char* p = static_cast<char*>(lm->weight_slab);
  lm->layers.resize(lm->L);
  for (int l = 0; l < lm->L; ++l) {
    LmLayer& w = lm->layers[l];
    w.wqkv = reinterpret_cast<uint16_t*>(p); p += (size_t)(lm->qs + 2 * lm->ks) * H * 2;
    w.wo = reinterpret_cast<uint16_t*>(p); p += H * lm->qs * 2;
    w.wgu = reinterpret_cast<uint16_t*>(p); p += 2 * I * H * 2;
    w.wd = reinterpret_cast<uint16_t*>(p); p += H * I * 2;
    w.ln_in = reinterpret_cast<float*>(p); p += H * 4;
    w.ln_post = reinterpret_cast<float*>(p); p += H * 4;
  }
  const size_t kv_bytes = (size_t)std::max(1, lm->L) * lm->kv_layer_stride() * 4;
  bool ok = cudaMalloc(&lm->norm_w, H * 4) == cudaSuccess &&
            cudaMalloc(&lm->kcache, kv_bytes) == cudaSuccess && cudaMalloc(&lm->vcache, kv_bytes) == cudaSuccess &&
            cudaMemset(lm->kcache, 0, kv_bytes) == cudaSuccess && cudaMemset(lm->vcache, 0, kv_bytes) == cudaSuccess &&
            cudaMalloc(&lm->d_pos, 64) == cudaSuccess && cudaMalloc(&lm->d_step, 64) == cudaSuccess &&
            cudaMalloc(&lm->d_tokens, (size_t)(max_length + 8) * 4) == cudaSuccess &&
            cudaMalloc(&lm->x, H * 4 * max_batch) == cudaSuccess && cudaMalloc(&lm->hid_norm, H * 4) == cudaSuccess &&
            cudaMalloc(&lm->q, lm->qs * 4 * max_batch) == cudaSuccess &&
            cudaMalloc(&lm->attn, lm->qs * 4 * max_batch) == cudaSuccess && cudaMalloc(&lm->act, I * 4 * max_batch) == cudaSuccess &&
            cudaMalloc(&lm->attn_partials, (size_t)max_batch * lm->nkv * 32 * lm->nh / lm->nkv * (d + 2) * 4) == cudaSuccess &&
            cudaMalloc(&lm->attn_counters, (size_t)max_batch * lm->nkv * 4) == cudaSuccess &&
            cudaMemset(lm->attn_counters, 0, (size_t)max_batch * lm->nkv * 4) == cudaSuccess &&
            cudaMalloc(&lm->argmax_partials, 4096 * sizeof(float2)) == cudaSuccess &&
            cudaMalloc(&lm->argmax_counter, 64) == cudaSuccess && cudaMemset(lm->argmax_counter, 0, 64) == cudaSuccess &&
            cudaMemset(lm->d_pos, 0, 64) == cudaSuccess && cudaMemset(lm->d_step, 0, 64) == cudaSuccess;
  if (ok && lm->V > 0) {
    ok = cudaMalloc(&lm->embed, (size_t)lm->V * H * 2) == cudaSuccess &&
         cudaMalloc(&lm->logits, (size_t)lm->V * 4) == cudaSuccess;
  }
  if (!ok) {
    cudaGetLastError();
    return fail_free(VX_ERR_OOM, "model buffer allocation failed");
  }
  if (workspace_init(ctx, &lm->ws, std::max({lm->qs + 2 * lm->ks, 2 * lm->I, lm->H}),
                     std::max({lm->H, lm->I, lm->qs})) != VX_OK)
    return fail_free(VX_ERR_OOM, "linear workspace allocation failed");
  if (ctx->persist && lm->L > 0 && lm->embed &&
      persist_supported(lm->L, lm->H, lm->I, lm->nh, lm->nkv, d, lm->V, max_length)) {
    const int grid = persist_configure(lm->H, lm->I, lm->nh, lm->nkv, d, max_length, ctx->persist_nst, ctx->persist_grid);
    if (grid > 0) {
      std::vector<PersistLayer> pl(lm->L);
      const size_t nc = persist_counter_count(lm->L);
      ok = cudaMalloc(&lm->pk_wdt, (size_t)lm->L * I * H * 2) == cudaSuccess &&
           cudaMalloc(&lm->pk_xacc, 2 * H * 8) == cudaSuccess;
      for (int l = 0; ok && l < lm->L; ++l)
        pl[l] = {lm->layers[l].wqkv, lm->layers[l].wo, lm->layers[l].wgu, lm->pk_wdt + (size_t)l * I * H,
                 lm->layers[l].ln_in, lm->layers[l].ln_post};
      ok = ok && cudaMalloc(&lm->x_mid, H * 4) == cudaSuccess &&
           cudaMalloc(&lm->pk_layers, sizeof(PersistLayer) * lm->L) == cudaSuccess &&
           cudaMemcpy(lm->pk_layers, pl.data(), sizeof(PersistLayer) * lm->L, cudaMemcpyHostToDevice) == cudaSuccess &&
           cudaMalloc(&lm->pk_cnt, nc * 4) == cudaSuccess && cudaMemset(lm->pk_cnt, 0, nc * 4) == cudaSuccess &&
           cudaMalloc(&lm->pk_att_part, persist_att_global_floats(lm->nkv, lm->nh, d) * 4) == cudaSuccess &&
           cudaMemset(lm->pk_att_part, 0, persist_att_global_floats(lm->nkv, lm->nh, d) * 4) == cudaSuccess;
      if (!ok) {
        cudaGetLastError();
        return fail_free(VX_ERR_OOM, "persistent decode buffers allocation failed");
      }
      lm->pk_grid = grid;
    }
  }
  *out = lm;
  return VX_OK;
}

void vx_lm_destroy(vx_lm* lm) {
  if (!lm) return;
  cudaSetDevice(lm->ctx->device);
  cudaStreamSynchronize(lm->ctx->stream);
  if (lm->step_exec) cudaGraphExecDestroy(lm->step_exec);
  for (auto& e : lm->ev)
    if (e) cudaEventDestroy(e);
  free_prefill(lm);
  workspace_free(&lm->ws);
  if (lm->bstep_exec) cudaGraphExecDestroy(lm->bstep_exec);
  persist_stack_free(lm->bp);
  for (void* p : {(void*)lm->bx, (void*)lm->bxn, (void*)lm->bqkv, (void*)lm->bq, (void*)lm->battn, (void*)lm->bgu,
                  (void*)lm->bact, (void*)lm->blogits, (void*)lm->bhid, (void*)lm->btokens})
    if (p) cudaFree(p);
  void* ptrs[] = {lm->weight_slab, lm->norm_w, lm->embed, lm->rope, lm->rope_tab, lm->kcache, lm->vcache, lm->d_pos,
                  lm->d_step, lm->d_tokens, lm->x, lm->hid_norm, lm->q, lm->attn, lm->act, lm->logits,
                  lm->attn_partials,
                  lm->attn_counters, lm->argmax_partials, lm->argmax_counter, lm->pf_ids,
                  lm->x_mid,         lm->pk_layers, lm->pk_cnt, lm->pk_att_part, lm->pk_xacc, lm->pk_wdt};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  delete lm;
}

int vx_lm_load_layer(vx_lm* lm, int layer, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                     const uint16_t* o, const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                     const float* ln_in, const float* ln_post) {
  if (!lm || !q || !k || !v || !o || !gate || !up || !down || !ln_in || !ln_post) return VX_ERR_ARG;
  if (layer < 0 || layer >= lm->L) return fail(lm->ctx, VX_ERR_ARG, "layer %d out of range", layer);
  vx_ctx* ctx = lm->ctx;
  cudaSetDevice(ctx->device);
  const LmLayer& w = lm->layers[layer];
  const size_t H = lm->H, I = lm->I;
  cudaStream_t st = ctx->stream;
  // fuse_qkv / fuse_gate_up (weights.rs:648-772): row-major [out, in] concat along out
  VX_CUDA(ctx, cudaMemcpyAsync(w.wqkv, q, (size_t)lm->qs * H * 2, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.wqkv + (size_t)lm->qs * H, k, (size_t)lm->ks * H * 2, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.wqkv + (size_t)(lm->qs + lm->ks) * H, v, (size_t)lm->ks * H * 2, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.wo, o, H * lm->qs * 2, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.wgu, gate, I * H * 2, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.wgu + I * H, up, I * H * 2, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.wd, down, H * I * 2, cudaMemcpyDefault, st));
  // the persistent step streams down_proj as rows of its transpose (one contiguous 8-row
  // group per MLP unit)
  if (lm->pk_wdt) VX_CUDA(ctx, transpose_bf16(w.wd, lm->pk_wdt + (size_t)layer * I * H, (int)H, (int)I, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.ln_in, ln_in, H * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaMemcpyAsync(w.ln_post, ln_post, H * 4, cudaMemcpyDefault, st));
  VX_CUDA(ctx, cudaStreamSynchronize(st));
  return VX_OK;
}

int vx_lm_load_norm(vx_lm* lm, const float* w) {
  if (!lm || !w) return VX_ERR_ARG;
  cudaSetDevice(lm->ctx->device);
  VX_CUDA(lm->ctx, cudaMemcpy(lm->norm_w, w, (size_t)lm->H * 4, cudaMemcpyDefault));
  return VX_OK;
}

int vx_lm_load_embed(vx_lm* lm, const uint16_t* embed) {
  if (!lm || !embed) return VX_ERR_ARG;
  if (!lm->embed) return fail(lm->ctx, VX_ERR_CONFIG, "model has no vocabulary");
  cudaSetDevice(lm->ctx->device);
  VX_CUDA(lm->ctx, cudaMemcpy(lm->embed, embed, (size_t)lm->V * lm->H * 2, cudaMemcpyDefault));
  return VX_OK;
}

int vx_lm_reset(vx_lm* lm) {
  if (!lm) return VX_ERR_ARG;
  lm->cur_len = 0;
  return VX_OK;
}

int vx_lm_position(const vx_lm* lm) { return lm ? lm->cur_len : -1; }

int vx_lm_set_position(vx_lm* lm, int pos) {
  if (!lm) return VX_ERR_ARG;
  if (pos < 0 || pos > lm->max_length) return fail(lm->ctx, VX_ERR_ARG, "position out of range");
  lm->cur_len = pos;
  return VX_OK;
}

int vx_lm_kv_write(vx_lm* lm, int layer, int b, const float* k, const float* v, int n_pos) {
  if (!lm || !k || !v) return VX_ERR_ARG;
  if (layer < 0 || layer >= lm->L || b < 0 || b >= lm->max_batch || n_pos < 0 || n_pos > lm->max_length)
    return fail(lm->ctx, VX_ERR_ARG, "kv_write: index out of range");
  cudaSetDevice(lm->ctx->device);
  const size_t row = (size_t)n_pos * lm->d * 4;
  for (int g = 0; g < lm->nkv; ++g) {
    VX_CUDA(lm->ctx, cudaMemcpy(lm->kc(layer, b) + (size_t)g * lm->max_length * lm->d, k + (size_t)g * n_pos * lm->d,
                                row, cudaMemcpyDefault));
    VX_CUDA(lm->ctx, cudaMemcpy(lm->vc(layer, b) + (size_t)g * lm->max_length * lm->d, v + (size_t)g * n_pos * lm->d,
                                row, cudaMemcpyDefault));
  }
  return VX_OK;
}

int vx_lm_kv_read(vx_lm* lm, int layer, int b, float* k, float* v, int n_pos) {
  if (!lm || !k || !v) return VX_ERR_ARG;
  if (layer < 0 || layer >= lm->L || b < 0 || b >= lm->max_batch || n_pos < 0 || n_pos > lm->max_length)
    return fail(lm->ctx, VX_ERR_ARG, "kv_read: index out of range");
  cudaSetDevice(lm->ctx->device);
  VX_CUDA(lm->ctx, cudaStreamSynchronize(lm->ctx->stream));
  const size_t row = (size_t)n_pos * lm->d * 4;
  for (int g = 0; g < lm->nkv; ++g) {
    VX_CUDA(lm->ctx, cudaMemcpy(k + (size_t)g * n_pos * lm->d, lm->kc(layer, b) + (size_t)g * lm->max_length * lm->d,
                                row, cudaMemcpyDefault));
    VX_CUDA(lm->ctx, cudaMemcpy(v + (size_t)g * n_pos * lm->d, lm->vc(layer, b) + (size_t)g * lm->max_length * lm->d,
                                row, cudaMemcpyDefault));
  }
  return VX_OK;
}

int vx_lm_embed(vx_lm* lm, const int32_t* ids, int n, float* out) {
  if (!lm || !ids || !out || n <= 0) return VX_ERR_ARG;
  if (!lm->embed) return fail(lm->ctx, VX_ERR_CONFIG, "model has no vocabulary");
  cudaSetDevice(lm->ctx->device);
  VX_CUDA(lm->ctx, launch_embed(lm->embed, ids, n, lm->H, lm->V, lm->emb_scale, out, lm->ctx->stream));
  return VX_OK;
}

int vx_lm_forward(vx_lm* lm, const float* embeds, int B, int S, int causal, int fill_cache, float* hidden_out) {
  if (!lm || !embeds || !hidden_out) return VX_ERR_ARG;
  vx_ctx* ctx = lm->ctx;
  if (B <= 0 || S <= 0) return fail(ctx, VX_ERR_SHAPE, "forward: empty input");
  if (fill_cache && (B > lm->max_batch || S > lm->max_length))
    return fail(ctx, VX_ERR_KV_FULL, "forward: %d positions exceed the cache (%d)", S, lm->max_length);
  cudaSetDevice(ctx->device);
  const size_t M = (size_t)B * S;
  int rc = ensure_prefill(lm, M, B, S, !fill_cache);
  if (rc) return rc;
  cudaStream_t st = ctx->stream;
  const int H = lm->H, I = lm->I, qkvw = lm->qs + 2 * lm->ks;
  VX_CUDA(ctx, cudaMemcpyAsync(lm->pf_x, embeds, M * H * 4, cudaMemcpyDefault, st));
  // the RMSNorm, attention and SiLU*up kernels write the few-row GEMMs' split operand
  // themselves when the rows fit one tcgen05 chunk (the attention only as one launch)
  uint16_t* xs = lm->ws.scratch ? tc_gemm_presplit_buffer(lm->ws.scratch) : nullptr;
  const int Mi = (int)M;
  const bool ps_qkv = presplit_ok(ctx, &lm->ws, Mi, qkvw, H), ps_gu = presplit_ok(ctx, &lm->ws, Mi, 2 * I, H),
             ps_d = presplit_ok(ctx, &lm->ws, Mi, H, I),
             ps_o = presplit_ok(ctx, &lm->ws, Mi, H, lm->qs) && (!fill_cache || B == 1);
  const bool rope_in_att = !fill_cache && ctx->att_rope_fused && S <= ATT_FUSED_ROPE_MAX_S;
  for (int l = 0; l < lm->L; ++l) {
    const LmLayer& w = lm->layers[l];
    // K/V for this layer: the cache itself (prefill) or a [B, nkv, S, d] temporary
    float* kd = fill_cache ? lm->kc(l, 0) : lm->pf_k;
    float* vd = fill_cache ? lm->vc(l, 0) : lm->pf_v;
    const int s_max = fill_cache ? lm->max_length : S;
    VX_CUDA(ctx, launch_rmsnorm_residual(lm->pf_x, nullptr, w.ln_in, 1.f, lm->cfg.rms_norm_eps, Mi, H, nullptr,
                                         ps_qkv ? nullptr : lm->pf_xn, st, ps_qkv ? xs : nullptr));
    rc = ps_qkv ? linear_presplit(ctx, &lm->ws, Mi, qkvw, H, w.wqkv, nullptr, nullptr, 1.f, lm->pf_qkv, qkvw, st)
                : linear(ctx, &lm->ws, lm->pf_xn, H, Mi, qkvw, H, w.wqkv, nullptr, nullptr, 1.f, lm->pf_qkv, qkvw, st);
    if (rc) return rc;
    if (fill_cache) {
      for (int b = 0; b < B; ++b)
        VX_CUDA(ctx, launch_rope_scatter(lm->pf_qkv + (size_t)b * S * qkvw, 1, S, lm->nh, lm->nkv, lm->d, lm->rope, 0,
                                         lm->pf_q + (size_t)b * S * lm->qs, lm->kc(l, b), lm->vc(l, b), lm->max_length,
                                         st));
    } else if (!rope_in_att) {
      VX_CUDA(ctx, launch_rope_scatter(lm->pf_qkv, B, S, lm->nh, lm->nkv, lm->d, lm->rope, 0, lm->pf_q, kd, vd, S, st));
    }
    if (fill_cache) {
      for (int b = 0; b < B; ++b) {
        AttnPrefillArgs ap = {lm->pf_q + (size_t)b * S * lm->qs, lm->kc(l, b), lm->vc(l, b), 1, S, lm->nh, lm->nkv,
                              lm->d, s_max, lm->attn_scale, causal, lm->pf_attn + (size_t)b * S * lm->qs,
                              ps_o ? xs : nullptr, nullptr, nullptr};
        VX_CUDA(ctx, launch_attn_prefill(ap, st, true));
      }
    } else {
      // few rows without a cache (the DiT and LocEnc stacks): q / k rotated as the attention
      // loads them from the fused projection, no separate RoPE pass
      AttnPrefillArgs ap = {lm->pf_q, kd, vd, B, S, lm->nh, lm->nkv, lm->d, s_max, lm->attn_scale, causal, lm->pf_attn,
                            ps_o ? xs : nullptr, rope_in_att ? lm->pf_qkv : nullptr,
                            rope_in_att ? lm->rope_tab : nullptr};
      VX_CUDA(ctx, launch_attn_prefill(ap, st, true));
    }
    rc = ps_o ? linear_presplit(ctx, &lm->ws, Mi, H, lm->qs, w.wo, nullptr, lm->pf_x, lm->res_scale, lm->pf_x, H, st)
              : linear(ctx, &lm->ws, lm->pf_attn, lm->qs, Mi, H, lm->qs, w.wo, nullptr, lm->pf_x, lm->res_scale, lm->pf_x,
                       H, st);
    if (rc) return rc;
    VX_CUDA(ctx, launch_rmsnorm_residual(lm->pf_x, nullptr, w.ln_post, 1.f, lm->cfg.rms_norm_eps, Mi, H, nullptr,
                                         ps_gu ? nullptr : lm->pf_xn, st, ps_gu ? xs : nullptr));
    rc = ps_gu ? linear_presplit(ctx, &lm->ws, Mi, 2 * I, H, w.wgu, nullptr, nullptr, 1.f, lm->pf_gu, 2 * I, st)
               : linear(ctx, &lm->ws, lm->pf_xn, H, Mi, 2 * I, H, w.wgu, nullptr, nullptr, 1.f, lm->pf_gu, 2 * I, st);
    if (rc) return rc;
    VX_CUDA(ctx, launch_silu_mul(lm->pf_gu, Mi, I, lm->pf_act, st, ps_d ? xs : nullptr));
    rc = ps_d ? linear_presplit(ctx, &lm->ws, Mi, H, I, w.wd, nullptr, lm->pf_x, lm->res_scale, lm->pf_x, H, st)
              : linear(ctx, &lm->ws, lm->pf_act, I, Mi, H, I, w.wd, nullptr, lm->pf_x, lm->res_scale, lm->pf_x, H, st);
    if (rc) return rc;
  }
  VX_CUDA(ctx, launch_rmsnorm_residual(lm->pf_x, nullptr, lm->norm_w, 1.f, lm->cfg.rms_norm_eps, (int)M, H, nullptr,
                                       hidden_out, st));
  if (fill_cache) lm->cur_len = S;
  return VX_OK;
}

int vx_lm_layer_forward_step(vx_lm* lm, int layer, float* hidden, int pos) {
  if (!lm || !hidden) return VX_ERR_ARG;
  vx_ctx* ctx = lm->ctx;
  if (layer < 0 || layer >= lm->L) return fail(ctx, VX_ERR_ARG, "layer %d out of range", layer);
  if (pos < 0 || pos >= lm->max_length) return fail(ctx, VX_ERR_KV_FULL, "KV cache is full");
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  if (hidden != lm->x) VX_CUDA(ctx, cudaMemcpyAsync(lm->x, hidden, (size_t)lm->H * 4, cudaMemcpyDefault, st));
  int rc = enqueue_layer_step(lm, layer, st, false, pos);
  if (rc) return rc;
  if (hidden != lm->x) VX_CUDA(ctx, cudaMemcpyAsync(hidden, lm->x, (size_t)lm->H * 4, cudaMemcpyDefault, st));
  return VX_OK;
}

int vx_lm_forward_step(vx_lm* lm, const float* embeds, float* hidden_out) {
  if (!lm || !embeds || !hidden_out) return VX_ERR_ARG;
  vx_ctx* ctx = lm->ctx;
  // StaticKvCache::step (cache.rs:60-65)
  if (!(lm->cur_len < lm->max_length)) return fail(ctx, VX_ERR_KV_FULL, "KV cache is full");
  const int pos = lm->cur_len;
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  VX_CUDA(ctx, cudaMemcpyAsync(lm->x, embeds, (size_t)lm->H * 4, cudaMemcpyDefault, st));
  for (int l = 0; l < lm->L; ++l) {
    int rc = enqueue_layer_step(lm, l, st, false, pos);
    if (rc) return rc;
  }
  VX_CUDA(ctx, launch_rmsnorm_residual(lm->x, nullptr, lm->norm_w, 1.f, lm->cfg.rms_norm_eps, 1, lm->H, nullptr,
                                       hidden_out, st));
  lm->cur_len = pos + 1;
  return VX_OK;
}

}  // extern "C"

namespace vx {

vx_ctx* lm_ctx(vx_lm* lm) { return lm->ctx; }
const LinearWorkspace* lm_workspace(const vx_lm* lm) { return &lm->ws; }
int lm_prepare_rows(vx_lm* lm, size_t rows) { return ensure_prefill(lm, rows, 1, (int)rows, false); }
int lm_hidden_size(const vx_lm* lm) { return lm->H; }
const float* lm_hid_norm(const vx_lm* lm) { return lm->hid_norm; }

// Validate, prefill the prompt (causal forward + cache fill), pick the first id with the
// greedy head and set the device position for the decode steps.  Records ev[0], ev[1].
int lm_greedy_begin(vx_lm* lm, const int32_t* prompt_ids, int n_prompt, int n_steps) {
  vx_ctx* ctx = lm->ctx;
  if (!lm->embed) return fail(ctx, VX_ERR_CONFIG, "greedy decode needs a vocabulary");
  if (n_prompt + n_steps > lm->max_length)
    return fail(ctx, VX_ERR_KV_FULL, "KV cache is full: %d prompt + %d steps > %d", n_prompt, n_steps, lm->max_length);
  for (int i = 0; i < n_prompt; ++i)
    if (prompt_ids[i] < 0 || prompt_ids[i] >= lm->V)
      return fail(ctx, VX_ERR_ARG, "prompt id %d at %d outside the vocabulary", prompt_ids[i], i);
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  if (lm->pf_ids_cap < n_prompt) {
    if (lm->pf_ids) cudaFree(lm->pf_ids);
    lm->pf_ids = nullptr;
    lm->pf_ids_cap = 0;
    VX_CUDA(ctx, cudaMalloc(&lm->pf_ids, (size_t)n_prompt * 4));
    lm->pf_ids_cap = n_prompt;
  }
  int rc = ensure_prefill(lm, n_prompt, 1, n_prompt, false);
  if (rc) return rc;
  if (!lm->ev[0])
    for (auto& e : lm->ev) VX_CUDA(ctx, cudaEventCreate(&e));
  rc = build_step_graph(lm);
  if (rc) return rc;
  VX_CUDA(ctx, cudaEventRecord(lm->ev[0], st));
  if (lm->pk_cnt) {
    VX_CUDA(ctx, cudaMemsetAsync(lm->pk_cnt, 0, persist_counter_count(lm->L) * 4, st));
    // the attention arrival counters behind the split partials and the merged output
    const size_t off = persist_att_partials_floats(lm->nkv, lm->nh, lm->d) + (size_t)lm->nh * lm->d;
    VX_CUDA(ctx, cudaMemsetAsync(lm->pk_att_part + off, 0, (size_t)lm->nkv * 4, st));
  }
  VX_CUDA(ctx, cudaMemsetAsync(lm->attn_counters, 0, (size_t)lm->max_batch * lm->nkv * 4, st));
  VX_CUDA(ctx, cudaMemsetAsync(lm->argmax_counter, 0, 4, st));
  // prefill: embed * scale_emb -> causal forward -> StaticKvCache::fill (voxcpm2/model.rs:144-191)
  VX_CUDA(ctx, cudaMemcpyAsync(lm->pf_ids, prompt_ids, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, st));
  VX_CUDA(ctx, launch_embed(lm->embed, lm->pf_ids, n_prompt, lm->H, lm->V, lm->emb_scale, lm->pf_xn, st));
  // vx_lm_forward consumes the embeddings through its own copy; pf_xn is only the source
  rc = vx_lm_forward(lm, lm->pf_xn, 1, n_prompt, 1, 1, lm->pf_gu);
  if (rc) return rc;
  // The last un-normed hidden row feeds the LM head, which applies the final norm itself.
  VX_CUDA(ctx, cudaMemcpyAsync(lm->x, lm->pf_x + (size_t)(n_prompt - 1) * lm->H, (size_t)lm->H * 4,
                               cudaMemcpyDeviceToDevice, st));
  VX_CUDA(ctx, cudaMemsetAsync(lm->d_step, 0, 4, st));
  rc = enqueue_lm_head(lm, st, false, n_steps == 0);
  if (rc) return rc;
  lm->pos_host = n_prompt;
  VX_CUDA(ctx, cudaMemcpyAsync(lm->d_pos, &lm->pos_host, 4, cudaMemcpyHostToDevice, st));
  VX_CUDA(ctx, cudaEventRecord(lm->ev[1], st));
  lm->cur_len = n_prompt;
  return VX_OK;
}

// Batched greedy start for B prompts of equal length (ids [B][n_prompt]): causal prefill of
// all rows filling the cache rows 0..B-1, then the head picks each row's first id.
int lm_batch_begin(vx_lm* lm, const int32_t* prompt_ids, int B, int n_prompt, int n_steps) {
  vx_ctx* ctx = lm->ctx;
  if (!lm->embed) return fail(ctx, VX_ERR_CONFIG, "greedy decode needs a vocabulary");
  if (B <= 0 || B > lm->max_batch) return fail(ctx, VX_ERR_SHAPE, "batch %d outside 1..%d", B, lm->max_batch);
  if (B > 128) return fail(ctx, VX_ERR_SHAPE, "batch %d > 128", B);
  if (n_prompt + n_steps > lm->max_length)
    return fail(ctx, VX_ERR_KV_FULL, "KV cache is full: %d prompt + %d steps > %d", n_prompt, n_steps, lm->max_length);
  for (int i = 0; i < B * n_prompt; ++i)
    if (prompt_ids[i] < 0 || prompt_ids[i] >= lm->V)
      return fail(ctx, VX_ERR_ARG, "prompt id %d at %d outside the vocabulary", prompt_ids[i], i);
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  int rc = ensure_batch(lm);
  if (rc) return rc;
  const int rows = B * n_prompt;
  if (lm->pf_ids_cap < rows) {
    if (lm->pf_ids) cudaFree(lm->pf_ids);
    lm->pf_ids = nullptr;
    lm->pf_ids_cap = 0;
    VX_CUDA(ctx, cudaMalloc(&lm->pf_ids, (size_t)rows * 4));
    lm->pf_ids_cap = rows;
  }
  if ((rc = ensure_prefill(lm, rows, B, n_prompt, false))) return rc;
  if ((rc = build_batch_graph(lm, B))) return rc;
  VX_CUDA(ctx, cudaMemsetAsync(lm->attn_counters, 0, (size_t)lm->max_batch * lm->nkv * 4, st));
  VX_CUDA(ctx, cudaMemcpyAsync(lm->pf_ids, prompt_ids, (size_t)rows * 4, cudaMemcpyHostToDevice, st));
  VX_CUDA(ctx, launch_embed(lm->embed, lm->pf_ids, rows, lm->H, lm->V, lm->emb_scale, lm->pf_xn, st));
  if ((rc = vx_lm_forward(lm, lm->pf_xn, B, n_prompt, 1, 1, lm->pf_gu))) return rc;
  // each row's last un-normed hidden feeds the head
  VX_CUDA(ctx, cudaMemcpy2DAsync(lm->bx, (size_t)lm->H * 4, lm->pf_x + (size_t)(n_prompt - 1) * lm->H,
                                 (size_t)n_prompt * lm->H * 4, (size_t)lm->H * 4, B, cudaMemcpyDeviceToDevice, st));
  VX_CUDA(ctx, cudaMemsetAsync(lm->d_step, 0, 4, st));
  if ((rc = enqueue_batch_head(lm, B, st, false))) return rc;
  lm->pos_host = n_prompt;
  VX_CUDA(ctx, cudaMemcpyAsync(lm->d_pos, &lm->pos_host, 4, cudaMemcpyHostToDevice, st));
  lm->cur_len = n_prompt;
  return VX_OK;
}

// One graph-replayed batched decode step (B rows as at lm_batch_begin).
int lm_batch_step(vx_lm* lm) {
  vx_ctx* ctx = lm->ctx;
  if (!(lm->cur_len < lm->max_length)) return fail(ctx, VX_ERR_KV_FULL, "KV cache is full");
  VX_CUDA(ctx, cudaGraphLaunch(lm->bstep_exec, ctx->stream));
  count_launch(lm->bstep_kernels);
  lm->cur_len += 1;
  return VX_OK;
}

const float* lm_batch_hidden(const vx_lm* lm) { return lm->bhid; }
const int* lm_batch_tokens(const vx_lm* lm) { return lm->btokens; }
int lm_max_batch(const vx_lm* lm) { return lm->max_batch; }
int lm_vocab_size(const vx_lm* lm) { return lm->V; }
void lm_stack_view(const vx_lm* lm, LmStackView* v) {
  v->L = lm->L;
  v->H = lm->H;
  v->I = lm->I;
  v->nh = lm->nh;
  v->nkv = lm->nkv;
  v->d = lm->d;
  v->eps = lm->cfg.rms_norm_eps;
  v->res_scale = lm->res_scale;
  v->attn_scale = lm->attn_scale;
  v->rope = lm->rope;
  v->norm_w = lm->norm_w;
  v->layers.resize(lm->L);
  for (int l = 0; l < lm->L; ++l) {
    const LmLayer& w = lm->layers[l];
    v->layers[l] = {w.wqkv, w.wo, w.wgu, w.wd, w.ln_in, w.ln_post};
  }
}
void lm_dims(const vx_lm* lm, int* L, int* H, int* I, int* qs, int* ks, int* V) {
  *L = lm->L;
  *H = lm->H;
  *I = lm->I;
  *qs = lm->qs;
  *ks = lm->ks;
  *V = lm->V;
}
int lm_max_length(const vx_lm* lm) { return lm->max_length; }

// One graph-replayed decode step: consumes the last picked id at the device position,
// writes the next id, the final-norm hidden (hid_norm) and advances the position.
int lm_greedy_step(vx_lm* lm) {
  vx_ctx* ctx = lm->ctx;
  if (!(lm->cur_len < lm->max_length)) return fail(ctx, VX_ERR_KV_FULL, "KV cache is full");
  VX_CUDA(ctx, cudaGraphLaunch(lm->step_exec, ctx->stream));
  count_launch(lm->step_kernels);
  lm->cur_len += 1;
  return VX_OK;
}

}  // namespace vx

extern "C" {

int vx_lm_batch_trace(vx_lm* lm, unsigned long long* out, int n, int* grid, int* phases) {
  if (!lm || !out || !grid || !phases || !lm->bp.trace) return VX_ERR_ARG;
  *grid = lm->bp.grid;
  *phases = 8 * lm->L + 1;
  const size_t need = (size_t)*grid * *phases * 4;
  if ((size_t)n < need) return VX_ERR_ARG;
  cudaSetDevice(lm->ctx->device);
  VX_CUDA(lm->ctx, cudaStreamSynchronize(lm->ctx->stream));
  VX_CUDA(lm->ctx, cudaMemcpy(out, lm->bp.trace, need * 8, cudaMemcpyDeviceToHost));
  return VX_OK;
}

int vx_lm_greedy(vx_lm* lm, const int32_t* prompt_ids, int n_prompt, int n_steps, int32_t* tokens_out) {
  if (!lm || !prompt_ids || !tokens_out || n_prompt <= 0 || n_steps < 0) return VX_ERR_ARG;
  vx_ctx* ctx = lm->ctx;
  int rc = lm_greedy_begin(lm, prompt_ids, n_prompt, n_steps);
  if (rc) return rc;
  cudaStream_t st = ctx->stream;
  const int pos0 = n_prompt;
  for (int s = 0; s < n_steps; ++s) {
    if (ctx->cancel.load(std::memory_order_relaxed)) {
      cudaStreamSynchronize(st);
      lm->cur_len = pos0 + s;
      return fail(ctx, VX_ERR_CANCELLED, "generation cancelled");
    }
    VX_CUDA(ctx, cudaGraphLaunch(lm->step_exec, st));
    count_launch(lm->step_kernels);
  }
  VX_CUDA(ctx, cudaEventRecord(lm->ev[2], st));
  VX_CUDA(ctx, cudaMemcpyAsync(tokens_out, lm->d_tokens, (size_t)(n_steps + 1) * 4, cudaMemcpyDeviceToHost, st));
  rc = check_device_error(ctx);
  if (rc) return rc;
  cudaEventElapsedTime(&lm->t_prefill_ms, lm->ev[0], lm->ev[1]);
  cudaEventElapsedTime(&lm->t_decode_ms, lm->ev[1], lm->ev[2]);
  lm->cur_len = pos0 + n_steps;
  return VX_OK;
}

int vx_lm_profile_decode_step(vx_lm* lm, int pos, float* kernel_us, int n) {
  if (!lm || !kernel_us) return VX_ERR_ARG;
  vx_ctx* ctx = lm->ctx;
  const int nk = lm->L * 5 + 1;
  if (n < nk) return fail(ctx, VX_ERR_ARG, "kernel_us needs %d entries", nk);
  if (pos < 0 || pos >= lm->max_length || !lm->embed) return fail(ctx, VX_ERR_ARG, "bad position or no vocabulary");
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  std::vector<cudaEvent_t> ev(nk + 1);
  for (auto& e : ev) VX_CUDA(ctx, cudaEventCreate(&e));
  const bool pdl = ctx->pdl;
  ctx->pdl = false;  // serialised: each kernel timed alone
  lm->pos_host = pos;
  VX_CUDA(ctx, cudaMemcpyAsync(lm->d_pos, &lm->pos_host, 4, cudaMemcpyHostToDevice, st));
  int rc = VX_OK;
  int k = 0;
  VX_CUDA(ctx, cudaEventRecord(ev[0], st));
  for (int l = 0; l < lm->L && !rc; ++l) {
    rc = enqueue_layer_step(lm, l, st, true, 0, &ev[k + 1]);  // one event after each launch
    k += 5;
  }
  if (!rc) rc = enqueue_lm_head(lm, st, false, false);
  VX_CUDA(ctx, cudaEventRecord(ev[++k], st));
  ctx->pdl = pdl;
  VX_CUDA(ctx, cudaStreamSynchronize(st));
  for (int i = 0; i < nk; ++i) kernel_us[i] = 0.f;
  for (int i = 0; i < k; ++i) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ev[i], ev[i + 1]);
    kernel_us[i] = ms * 1000.f;
  }
  for (auto& e : ev) cudaEventDestroy(e);
  return rc;
}

int vx_lm_trace_decode_step(vx_lm* lm, int pos, unsigned long long* trace_out, int n, int* grid_out) {
  if (!lm || !trace_out || !grid_out) return VX_ERR_ARG;
  vx_ctx* ctx = lm->ctx;
  if (lm->pk_grid <= 0) return fail(ctx, VX_ERR_CONFIG, "this model runs the per-kernel decode step");
  const size_t ne = persist_trace_entries(lm->L, lm->pk_grid);
  if ((size_t)n < ne) return fail(ctx, VX_ERR_ARG, "trace_out needs %zu entries", ne);
  if (pos < 0 || pos >= lm->max_length) return fail(ctx, VX_ERR_KV_FULL, "position out of range");
  cudaSetDevice(ctx->device);
  cudaStream_t st = ctx->stream;
  unsigned long long* dtrace = nullptr;
  VX_CUDA(ctx, cudaMalloc(&dtrace, ne * 8));
  int rc = VX_OK;
  lm->pos_host = pos;
  cudaError_t e = cudaMemsetAsync(dtrace, 0, ne * 8, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(lm->d_pos, &lm->pos_host, 4, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(lm->pk_cnt, 0, persist_counter_count(lm->L) * 4, st);
  if (e == cudaSuccess)
    e = cudaMemsetAsync(lm->pk_att_part + persist_att_partials_floats(lm->nkv, lm->nh, lm->d) + (size_t)lm->nh * lm->d,
                        0, (size_t)lm->nkv * 4, st);
  if (e == cudaSuccess) e = enqueue_persist_step(lm, st, true, dtrace);
  if (e == cudaSuccess) e = cudaMemcpyAsync(trace_out, dtrace, ne * 8, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) rc = cuda_fail(ctx, e, "trace decode step");
  cudaFree(dtrace);
  if (rc) return rc;
  *grid_out = lm->pk_grid;
  return check_device_error(ctx);
}

int vx_lm_last_timing(const vx_lm* lm, float* prefill_ms, float* decode_ms) {
  if (!lm || !prefill_ms || !decode_ms) return VX_ERR_ARG;
  *prefill_ms = lm->t_prefill_ms;
  *decode_ms = lm->t_decode_ms;
  return VX_OK;
}

int vx_lm_last_logits(vx_lm* lm, float* logits_out) {
  if (!lm || !logits_out) return VX_ERR_ARG;
  if (!lm->logits) return fail(lm->ctx, VX_ERR_CONFIG, "model has no vocabulary");
  cudaSetDevice(lm->ctx->device);
  VX_CUDA(lm->ctx, cudaStreamSynchronize(lm->ctx->stream));
  VX_CUDA(lm->ctx, cudaMemcpy(logits_out, lm->logits, (size_t)lm->V * 4, cudaMemcpyDeviceToHost));
  return VX_OK;
}

}  // extern "C"
