// C-ABI entry points for the norms, attention, glue and the whole denoise loop.
//
// pi05_denoise_step enqueues one Euler step of the action expert on a stream:
//   action_in_proj -> 18 x [QKV+RoPE+KV-tail (input adaRMS folded in), MQA
//   attention (+ split combine), o_proj+gated residual, gate/up+GeGLU
//   (post-attention adaRMS folded in), down+gated residual]
//   -> final adaRMS + action_out_proj + Euler update.
// Without folded weights (or with more than 64 tokens) the two adaRMS norms of a
// layer run as kernels of their own before the projections.
// Every launch carries the PDL attribute, so each kernel's prologue and weight
// prefetch overlap the previous kernel's tail.  The engine captures the whole
// loop in one CUDA graph.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "../../include/pi05_b200.h"
#include "attention.h"
#include "elementwise.h"
#include "host_util.h"
#include "skinny_gemm.h"

using namespace pi05;

namespace {

inline bool nz(const void* p) { return p != nullptr; }

// PI05_SPLITS="q,o,g,d" in the environment forces the split-K count of the four
// denoise GEMMs (tuning only; 0 or absent = automatic).
const int* debug_split_overrides() {
  static int v[4] = {0, 0, 0, 0};
  static bool init = [] {
    const char* e = getenv("PI05_SPLITS");
    if (e != nullptr) sscanf(e, "%d,%d,%d,%d", &v[0], &v[1], &v[2], &v[3]);
    return true;
  }();
  (void)init;
  return v;
}

// PI05_FOLD_NORM=0 in the environment keeps the norm kernels even when the plan
// carries folded weights (A/B and parity tests of the folded-norm path).
bool fold_norm_enabled() {
  static int v = [] {
    const char* e = getenv("PI05_FOLD_NORM");
    return (e != nullptr && e[0] == '0') ? 0 : 1;
  }();
  return v != 0;
}

}  // namespace

extern "C" {

int pi05_fold_adarms(const void* w, int rows, int k, const float* scale, const float* shift, void* w_out,
                     float* b_out, void* stream) {
  if (!nz(w) || !nz(scale) || !nz(shift) || !nz(w_out) || !nz(b_out)) {
    set_last_error("fold_adarms: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  return fold_adarms_run(w, rows, k, scale, shift, w_out, b_out, stream);
}

int pi05_rms_norm(const void* x, int ldx, const float* mod, const float* weight, void* out, int ldo, int rows, int d,
                  float eps, void* stream) {
  if (!nz(x) || !nz(out) || (!nz(mod) && !nz(weight))) {
    set_last_error("rms_norm: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  return rms_norm_run(x, ldx, mod, weight, out, ldo, rows, d, eps, stream);
}

int pi05_attention(const void* q, const void* k, const void* v, const uint8_t* key_valid, void* out, int rows,
                   int kv_len, int head_dim, float scale, int splits, void* workspace, size_t workspace_bytes,
                   void* stream) {
  if (!nz(q) || !nz(k) || !nz(v) || !nz(key_valid) || !nz(out)) {
    set_last_error("attention: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out)) {
    set_last_error("attention: pointers must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  Workspace w;
  if (split_workspace(workspace, workspace_bytes, &w)) {
    set_last_error("attention: workspace missing or too small");
    return PI05_ERR_WORKSPACE;
  }
  AttnParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride = head_dim;
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.kv_stride = head_dim;
  p.key_valid = key_valid;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_stride = head_dim;
  p.rows = rows;
  p.kv_len = kv_len;
  p.head_dim = head_dim;
  p.status = w.status;
  p.scale = scale;
  p.trace = debug_trace_buffer();
  return mqa_attention_run(p, w.scratch, w.scratch_bytes, splits, stream);
}

int pi05_action_in(const float* x, const float* w, const float* b, void* h, int rows, int din, int dout,
                   void* stream) {
  if (!nz(x) || !nz(w) || !nz(b) || !nz(h)) {
    set_last_error("action_in: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  return action_in_run(x, w, b, h, rows, din, dout, stream);
}

int pi05_final_euler(const void* h, const float* mod, const float* w, const float* b, float* x_t, float* v_out,
                     int rows, int d, int dout, float eps, float t, float delta, void* stream) {
  if (!nz(h) || !nz(mod) || !nz(w) || !nz(b) || !nz(x_t)) {
    set_last_error("final_euler: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  return final_euler_run(h, mod, w, b, x_t, v_out, rows, d, dout, eps, t, delta, stream);
}

int pi05_rope_table(const uint8_t* valid, int n_prefix, int mode, int rows, const float* inv_freq, int d, void* cos,
                    void* sin, void* stream) {
  if (!nz(valid) || !nz(inv_freq) || !nz(cos) || !nz(sin)) {
    set_last_error("rope_table: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  return rope_table_run(valid, n_prefix, mode, rows, inv_freq, d, cos, sin, stream);
}

int pi05_adarms_table(const float* timesteps, int n_steps, int width, const float* w_tin, const float* b_tin,
                      const float* w_tout, const float* b_tout, const float* w_dense, const float* b_dense,
                      int n_norm, float* table, void* workspace, size_t workspace_bytes, void* stream) {
  if (!nz(timesteps) || !nz(w_tin) || !nz(b_tin) || !nz(w_tout) || !nz(b_tout) || !nz(w_dense) || !nz(b_dense) ||
      !nz(table)) {
    set_last_error("adarms_table: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (n_steps <= 0 || n_steps > 16 || width <= 0 || width % 2) {
    set_last_error("adarms_table: n_steps in [1, 16], even width");
    return PI05_ERR_SHAPE;
  }
  Workspace w;
  if (split_workspace(workspace, workspace_bytes, &w) ||
      w.scratch_bytes < (size_t)3 * n_steps * width * sizeof(float)) {
    set_last_error("adarms_table: workspace too small");
    return PI05_ERR_WORKSPACE;
  }
  float* emb = w.scratch;
  float* h1 = emb + (size_t)n_steps * width;
  float* cond = h1 + (size_t)n_steps * width;
  int rc = sinusoid_run(timesteps, n_steps, width, 4e-3, 4.0, emb, stream);
  if (!rc) rc = linear_f32_rows_run(emb, n_steps, width, w_tin, b_tin, h1, width, 1, stream);
  if (!rc) rc = linear_f32_rows_run(h1, n_steps, width, w_tout, b_tout, cond, width, 1, stream);
  if (!rc) rc = linear_f32_rows_run(cond, n_steps, width, w_dense, b_dense, table, n_norm * 3 * width, 0, stream);
  return rc;
}

int pi05_denoise_step(const Pi05ExpertPlan* P, int step, void* stream) {
  if (!nz(P) || !nz(P->layers) || !nz(P->host_timesteps) || !nz(P->mod_table)) {
    set_last_error("denoise_step: null plan field");
    return PI05_ERR_INVALID_ARG;
  }
  if (step < 0 || step >= P->num_steps) {
    set_last_error("denoise_step: step %d out of range", step);
    return PI05_ERR_INVALID_ARG;
  }
  // Tt: tokens of one observation; T: rows of every GEMM (B observations stacked).
  const int Tt = P->tokens, W = P->width, F = P->mlp_dim, HQ = P->n_q_heads, HKV = P->n_kv_heads, D = P->head_dim;
  const int B = P->batch > 1 ? P->batch : 1;
  const int T = Tt * B;
  if (HKV != 1 || D != 256 || W % 128 || F % 128 || P->kv_rows < P->prefix_len + Tt) {
    set_last_error("denoise_step: unsupported shape (hkv=%d d=%d width=%d mlp=%d)", HKV, D, W, F);
    return PI05_ERR_SHAPE;
  }
  if (B > 1 && (P->kv_stage == nullptr || !aligned16(P->kv_stage) || B > 1024)) {
    set_last_error("denoise_step: batch %d needs a 16-byte aligned kv_stage (and at most 1024 observations)", B);
    return PI05_ERR_INVALID_ARG;
  }
  Workspace ws;
  if (split_workspace(P->workspace, P->workspace_bytes, &ws)) {
    set_last_error("denoise_step: workspace missing or too small");
    return PI05_ERR_WORKSPACE;
  }
  const int n_norm = 2 * P->depth + 1;
  const float* mods = P->mod_table + (size_t)step * n_norm * 3 * W;
  const int* so = debug_split_overrides();  // per GEMM (qkv, o, gate/up, down); 0 = automatic
  auto* h = static_cast<__nv_bfloat16*>(P->h);
  auto* xn = static_cast<__nv_bfloat16*>(P->xn);
  auto* q = static_cast<__nv_bfloat16*>(P->q);
  auto* attn = static_cast<__nv_bfloat16*>(P->attn);
  auto* act = static_cast<__nv_bfloat16*>(P->act);
  const int kv_len = P->prefix_len + Tt;
  // Batched: the q|k|v GEMM writes the new K / V rows to the staging buffer and a
  // scatter moves them to each observation's cache rows [prefix_len, prefix_len + Tt).
  auto* stage_k = static_cast<__nv_bfloat16*>(P->kv_stage);
  auto* stage_v = stage_k == nullptr ? nullptr : stage_k + (size_t)T * D;
  const float scale = 1.0f / std::sqrt((float)D);
  // Folded norms (default when the plan carries folded weights): no norm kernel
  // inside the layers.  action_in (layer 0) and down_proj write the row
  // statistics of input_layernorm's input to ssq_attn, o_proj those of
  // post_attention_layernorm's input to ssq_mlp; q|k|v and gate/up read h with the
  // step's folded weights and apply rstd and the folded bias to their accumulators.
  const int n_parts = W / 128;
  const bool fold = P->fold != nullptr && fold_norm_enabled() && n_parts <= kNormMaxParts &&
                    (size_t)2 * n_parts * T * sizeof(float) <= kWsStatsBytes;
  float* ssq_attn = ws.stats;
  float* ssq_mlp = ws.stats + (size_t)n_parts * T;
  const Pi05ExpertFold* FS = fold ? P->fold + (size_t)step * P->depth : nullptr;

  int rc = action_in_run(P->x_t, P->w_in, P->b_in, h, T, P->action_dim, W, stream, fold ? ssq_attn : nullptr, T);
  for (int l = 0; l < P->depth && rc == PI05_OK; ++l) {
    const Pi05ExpertLayer& L = P->layers[l];
    const float* mod1 = mods + (size_t)(2 * l) * 3 * W;
    const float* mod2 = mods + (size_t)(2 * l + 1) * 3 * W;
    // input_layernorm (adaRMS), unless folded into q|k|v
    if (!fold) {
      rc = rms_norm_run(h, W, mod1, nullptr, xn, W, T, W, P->eps, stream);
      if (rc) break;
    }
    // q|k|v + RoPE -> q, KV-cache tail rows [prefix_len, prefix_len + T)
    {
      SkinnyParams sp;
      sp.trace = P->trace;
      sp.status = ws.status;
      sp.counters = ws.counters;
      sp.accum = ws.accum;
      sp.accum_bytes = ws.accum_bytes;
      sp.m_tok = T;
      sp.allow_wide = 0;  // batched rows: 64-token tiles on blockIdx.y
      sp.max_tok = 64;
      sp.k = W;
      sp.n_tiles = (HQ + HKV) * (D / 128) + HKV * D / 128;
      sp.cos = static_cast<const __nv_bfloat16*>(P->rope_cos);
      sp.sin = static_cast<const __nv_bfloat16*>(P->rope_sin);
      sp.q_out = q;
      if (B > 1) {
        sp.k_cache = stage_k;
        sp.v_cache = stage_v;
        sp.kv_head_stride = (size_t)T * D;
        sp.krow0 = 0;
      } else {
        sp.k_cache = static_cast<__nv_bfloat16*>(L.k_cache);
        sp.v_cache = static_cast<__nv_bfloat16*>(L.v_cache);
        sp.kv_head_stride = (size_t)P->kv_rows * D;
        sp.krow0 = P->prefix_len;
      }
      sp.n_q_heads = HQ;
      sp.n_kv_heads = HKV;
      sp.head_dim = D;
      const int rows = (HQ + 2 * HKV) * D;
      sp.trace_tag = (step * P->depth + l) * 8 + 0;
      const void* wq = L.w_qkv;
      if (fold) {
        wq = FS[l].w_qkv;
        sp.fold_ssq = ssq_attn;
        sp.fold_parts = n_parts;
        sp.fold_ld = T;
        sp.fold_d = W;
        sp.fold_eps = P->eps;
        sp.fold_bias0 = FS[l].b_qkv;
        sp.fold_bias1 = FS[l].b_qkv;
      }
      rc = skinny_gemm_run(SK_EPI_QKV_ROPE, sp, wq, wq, rows, rows, fold ? h : xn, W, so[0], stream);
      if (rc) break;
      if (B > 1) {
        rc = kv_scatter_run(stage_k, stage_v, L.k_cache, L.v_cache, B, Tt, P->prefix_len, P->kv_rows, D, stream);
        if (rc) break;
      }
    }
    // attention over [prefix | suffix] keys
    {
      AttnParams ap;
      ap.q = q;
      ap.q_stride = D;
      ap.k = static_cast<const __nv_bfloat16*>(L.k_cache);
      ap.v = static_cast<const __nv_bfloat16*>(L.v_cache);
      ap.kv_stride = D;
      ap.key_valid = P->key_valid;
      ap.out = attn;
      ap.out_stride = D;
      ap.rows = Tt * HQ;
      ap.kv_len = kv_len;
      ap.batch = B;
      ap.q_batch = (size_t)Tt * HQ * D;
      ap.kv_batch = (size_t)P->kv_rows * D;
      ap.valid_batch = (size_t)P->kv_rows;
      ap.out_batch = (size_t)Tt * HQ * D;
      ap.head_dim = D;
      ap.scale = scale;
      ap.status = ws.status;
      ap.static_rows = P->prefix_len;  // prefix K/V rows and mask are fixed during the loop
      ap.trace = P->trace;
      ap.trace_tag = (step * P->depth + l) * 8 + 4;  // combine: + 5
      rc = mqa_attention_run(ap, ws.scratch, ws.scratch_bytes, P->attn_splits, stream);
      if (rc) break;
    }
    // o_proj + gated residual (gate = third chunk of mod1)
    {
      SkinnyParams sp;
      sp.trace = P->trace;
      sp.status = ws.status;
      sp.counters = ws.counters;
      sp.accum = ws.accum;
      sp.accum_bytes = ws.accum_bytes;
      sp.m_tok = T;
      sp.allow_wide = 0;  // batched rows: 64-token tiles on blockIdx.y
      sp.max_tok = 64;
      sp.k = HQ * D;
      sp.n_tiles = W / 128;
      sp.out = h;
      sp.ldo = W;
      sp.resid = h;
      sp.ldr = W;
      sp.gate = mod1 + 2 * W;
      sp.trace_tag = (step * P->depth + l) * 8 + 1;
      if (fold) {
        sp.row_ssq = ssq_mlp;
        sp.ssq_ld = T;
      }
      rc = skinny_gemm_run(SK_EPI_GATED_RESID, sp, L.w_o, L.w_o, W, W, attn, HQ * D, so[1], stream);
      if (rc) break;
    }
    // post_attention_layernorm (adaRMS), unless folded into gate/up
    if (!fold) {
      rc = rms_norm_run(h, W, mod2, nullptr, xn, W, T, W, P->eps, stream);
      if (rc) break;
    }
    // gate/up + GeGLU
    {
      SkinnyParams sp;
      sp.trace = P->trace;
      sp.status = ws.status;
      sp.counters = ws.counters;
      sp.accum = ws.accum;
      sp.accum_bytes = ws.accum_bytes;
      sp.m_tok = T;
      sp.allow_wide = 0;  // batched rows: 64-token tiles on blockIdx.y
      sp.max_tok = 64;
      sp.k = W;
      sp.n_tiles = F / 64;
      sp.out = act;
      sp.ldo = F;
      sp.trace_tag = (step * P->depth + l) * 8 + 2;
      const void* wg = L.w_gate;
      const void* wu = L.w_up;
      if (fold) {
        wg = FS[l].w_gate;
        wu = FS[l].w_up;
        sp.fold_ssq = ssq_mlp;
        sp.fold_parts = n_parts;
        sp.fold_ld = T;
        sp.fold_d = W;
        sp.fold_eps = P->eps;
        sp.fold_bias0 = FS[l].b_gate;
        sp.fold_bias1 = FS[l].b_up;
      }
      rc = skinny_gemm_run(SK_EPI_GEGLU, sp, wg, wu, F, F, fold ? h : xn, W, so[2], stream);
      if (rc) break;
    }
    // down + gated residual (gate = third chunk of mod2)
    {
      SkinnyParams sp;
      sp.trace = P->trace;
      sp.status = ws.status;
      sp.counters = ws.counters;
      sp.accum = ws.accum;
      sp.accum_bytes = ws.accum_bytes;
      sp.m_tok = T;
      sp.allow_wide = 0;  // batched rows: 64-token tiles on blockIdx.y
      sp.max_tok = 64;
      sp.k = F;
      sp.n_tiles = W / 128;
      sp.out = h;
      sp.ldo = W;
      sp.resid = h;
      sp.ldr = W;
      sp.gate = mod2 + 2 * W;
      if (fold && l + 1 < P->depth) {
        sp.row_ssq = ssq_attn;
        sp.ssq_ld = T;
      }
      sp.trace_tag = (step * P->depth + l) * 8 + 3;
      rc = skinny_gemm_run(SK_EPI_GATED_RESID, sp, L.w_down, L.w_down, W, W, act, F, so[3], stream);
      if (rc) break;
    }
  }
  if (rc) return rc;
  const float t = P->host_timesteps[step];
  const float delta = P->host_timesteps[step] - P->host_timesteps[step + 1];
  const float* coefs = P->host_step_coefs != nullptr ? P->host_step_coefs + 3 * step : nullptr;
  const float* noise = P->step_noise != nullptr ? P->step_noise + (size_t)step * T * P->action_dim : nullptr;
  return final_euler_run(h, mods + (size_t)(2 * P->depth) * 3 * W, P->w_out, P->b_out, P->x_t, P->v_t, T, W,
                         P->action_dim, P->eps, t, delta, stream, coefs, noise);
}

int pi05_denoise_loop(const Pi05ExpertPlan* plan, void* stream) {
  if (!nz(plan)) return PI05_ERR_INVALID_ARG;
  for (int s = 0; s < plan->num_steps; ++s) {
    int rc = pi05_denoise_step(plan, s, stream);
    if (rc) return rc;
  }
  return PI05_OK;
}

}  // extern "C"
