// Prefix LM (PaliGemma's Gemma-2B) with use_cache=True, and the language
// embedding gather.  The prefix forward writes each layer's rotated K and raw V
// straight into the expert's static KV buffers (rows [0, P)), so the reference's
// prime_kv_static copy (modeling_gemma.py:312-329) disappears.
//
// Per layer (transformers Gemma decoder, openpi-patched: no sqrt(width) input
// normaliser; q|k|v fused as in prefix_qkv_fused.py:132-139):
//   xn = RMSNorm(h) * (1 + w1)                        fp32 stats -> bf16
//   q, K, V = RoPE(xn @ Wqkv^T)                       K/V -> cache rows [0, P)
//   h = h + bf16(attn(q, K, V) @ Wo^T)                full attention among valid tokens
//   hn = RMSNorm(h) * (1 + w2)
//   h = h + bf16(GeGLU(hn) @ Wd^T)
// The last layer stops after K/V (prefix_last_layer.py:46-112).
#include <cmath>
#include <cstdlib>

#include "../../include/pi05_b200.h"
#include "attention.h"
#include "elementwise.h"
#include "host_util.h"
#include "ptx.cuh"
#include "skinny_gemm.h"

using namespace pi05;

namespace {

__global__ void __launch_bounds__(256) embed_tokens_kernel(const __nv_bfloat16* __restrict__ table, int vocab,
                                                           const int32_t* __restrict__ ids, int n, int d, float scale,
                                                           __nv_bfloat16* __restrict__ out, int ldo, int* status) {
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int row = blockIdx.x;
  const int id = ids[row];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) report_status(status, PI05_DEV_BAD_INDEX);
  for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
    __align__(16) __nv_bfloat16 o[8];
    if (ok) {
      const uint4 u = *reinterpret_cast<const uint4*>(table + (size_t)id * d + c);
      const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16(__bfloat162float(b[j]) * scale);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __float2bfloat16(0.f);
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * ldo + c) = *reinterpret_cast<const uint4*>(o);
  }
}

inline bool nz(const void* p) { return p != nullptr; }

// PI05_FOLD_NORM=0 in the environment keeps the RMSNorm kernels (A/B and parity
// tests of the folded path).
bool prefix_fold_enabled() {
  static int v = [] {
    const char* e = getenv("PI05_FOLD_NORM");
    return (e != nullptr && e[0] == '0') ? 0 : 1;
  }();
  return v != 0;
}

SkinnyParams base_params(const Workspace& ws) {
  SkinnyParams sp;
  sp.status = ws.status;
  sp.counters = ws.counters;
  sp.accum = ws.accum;
  sp.accum_bytes = ws.accum_bytes;
  sp.trace = debug_trace_buffer();
  return sp;
}

}  // namespace

extern "C" {

int pi05_embed_tokens(const void* table, int vocab, const int32_t* ids, int n, int d, float scale, void* out,
                      int ldo, void* workspace, size_t workspace_bytes, void* stream) {
  if (!nz(table) || !nz(ids) || !nz(out)) {
    set_last_error("embed_tokens: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (n <= 0 || d % 8 || ldo % 8 || !aligned16(table) || !aligned16(out)) {
    set_last_error("embed_tokens: need d, ldo multiples of 8 and 16-byte aligned table/out");
    return PI05_ERR_SHAPE;
  }
  Workspace ws;
  int* status = nullptr;
  if (workspace != nullptr && split_workspace(workspace, workspace_bytes, &ws) == PI05_OK) status = ws.status;
  return launch_pdl(embed_tokens_kernel, dim3(n), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                    pdl_enabled(), static_cast<const __nv_bfloat16*>(table), vocab, ids, n, d, scale,
                    static_cast<__nv_bfloat16*>(out), ldo, status);
}

int pi05_prefix_forward(const Pi05PrefixPlan* P, void* stream) {
  if (!nz(P) || !nz(P->layers) || !nz(P->key_valid) || !nz(P->inv_freq)) {
    set_last_error("prefix_forward: null plan field");
    return PI05_ERR_INVALID_ARG;
  }
  const int T = P->tokens, W = P->width, F = P->mlp_dim, HQ = P->n_q_heads, HKV = P->n_kv_heads, D = P->head_dim;
  if (HKV != 1 || D != 256 || W % 128 || F % 128 || T <= 0 || T > 4096 || P->kv_rows < T) {
    set_last_error("prefix_forward: unsupported shape (tokens=%d hkv=%d d=%d width=%d)", T, HKV, D, W);
    return PI05_ERR_SHAPE;
  }
  Workspace ws;
  if (split_workspace(P->workspace, P->workspace_bytes, &ws)) {
    set_last_error("prefix_forward: workspace missing or too small");
    return PI05_ERR_WORKSPACE;
  }
  auto* h = static_cast<__nv_bfloat16*>(P->h);
  auto* xn = static_cast<__nv_bfloat16*>(P->xn);
  auto* q = static_cast<__nv_bfloat16*>(P->q);
  auto* attn = static_cast<__nv_bfloat16*>(P->attn);
  auto* act = static_cast<__nv_bfloat16*>(P->act);
  const float scale = 1.0f / std::sqrt((float)D);

  // Folded norms: the RMSNorm weights (1 + w) live in folded copies of q|k|v and
  // gate/up; the residual GEMMs (o_proj, down_proj) write per-part sums of squares
  // of h to row_stats, and q|k|v / gate/up scale each token's accumulator by its
  // rstd (Gemma RMSNorm, fp32 statistics: modeling_gemma.py:94-99), so no norm
  // kernel runs.  The embeddings' statistics come from one row_ssq launch.
  bool fold = P->row_stats != nullptr && prefix_fold_enabled() && W <= 2048 && W % 64 == 0 &&
              row_ssq_parts(T, W) == W / 64;
  for (int l = 0; fold && l < P->depth; ++l)
    fold = nz(P->layers[l].wf_qkv) && nz(P->layers[l].wf_gate) && nz(P->layers[l].wf_up);
  const int parts = W / 64;
  auto fold_params = [&](SkinnyParams& sp) {
    sp.fold_ssq = P->row_stats;
    sp.fold_parts = parts;
    sp.fold_ld = T;
    sp.fold_d = W;
    sp.fold_eps = P->eps;
  };

  int rc = rope_table_run(P->key_valid, T, 0, T, P->inv_freq, D, P->rope_cos, P->rope_sin, stream);
  if (rc == PI05_OK && fold) rc = row_ssq_run(h, W, T, W, 64, P->row_stats, T, stream);
  for (int l = 0; l < P->depth && rc == PI05_OK; ++l) {
    const Pi05PrefixLayer& L = P->layers[l];
    const bool last = (l == P->depth - 1);
    if (!fold) rc = rms_norm_run(h, W, nullptr, L.ln1_w, xn, W, T, W, P->eps, stream);
    if (rc) break;
    {
      SkinnyParams sp = base_params(ws);
      sp.m_tok = T;
      sp.k = W;
      sp.n_tiles = (HQ + HKV) * (D / 128) + HKV * D / 128;
      sp.cos = static_cast<const __nv_bfloat16*>(P->rope_cos);
      sp.sin = static_cast<const __nv_bfloat16*>(P->rope_sin);
      sp.q_out = q;
      sp.k_cache = static_cast<__nv_bfloat16*>(L.k_cache);
      sp.v_cache = static_cast<__nv_bfloat16*>(L.v_cache);
      sp.kv_head_stride = (size_t)P->kv_rows * D;
      sp.krow0 = 0;
      sp.n_q_heads = HQ;
      sp.n_kv_heads = HKV;
      sp.head_dim = D;
      const int rows = (HQ + 2 * HKV) * D;
      if (fold) fold_params(sp);
      const void* wq = fold ? L.wf_qkv : L.w_qkv;
      rc = skinny_gemm_run(SK_EPI_QKV_ROPE, sp, wq, wq, rows, rows, fold ? h : xn, W, 0, stream);
      if (rc) break;
    }
    if (last && P->kv_only_last_layer) break;
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
      ap.rows = T * HQ;
      ap.kv_len = T;
      ap.head_dim = D;
      ap.status = ws.status;
      ap.scale = scale;
      rc = mqa_attention_run(ap, ws.scratch, ws.scratch_bytes, 0, stream);
      if (rc) break;
    }
    {
      SkinnyParams sp = base_params(ws);
      sp.m_tok = T;
      sp.k = HQ * D;
      sp.n_tiles = W / 128;
      sp.out = h;
      sp.ldo = W;
      sp.resid = h;
      sp.ldr = W;
      sp.gate = nullptr;
      if (fold) {
        sp.row_ssq = P->row_stats;
        sp.ssq_ld = T;
      }
      rc = skinny_gemm_run(SK_EPI_GATED_RESID, sp, L.w_o, L.w_o, W, W, attn, HQ * D, 0, stream);
      if (rc) break;
    }
    if (!fold) rc = rms_norm_run(h, W, nullptr, L.ln2_w, xn, W, T, W, P->eps, stream);
    if (rc) break;
    {
      SkinnyParams sp = base_params(ws);
      sp.m_tok = T;
      sp.k = W;
      sp.n_tiles = F / 64;
      sp.out = act;
      sp.ldo = F;
      if (fold) fold_params(sp);
      rc = skinny_gemm_run(SK_EPI_GEGLU, sp, fold ? L.wf_gate : L.w_gate, fold ? L.wf_up : L.w_up, F, F,
                           fold ? h : xn, W, 0, stream);
      if (rc) break;
    }
    {
      SkinnyParams sp = base_params(ws);
      sp.m_tok = T;
      sp.k = F;
      sp.n_tiles = W / 128;
      sp.out = h;
      sp.ldo = W;
      sp.resid = h;
      sp.ldr = W;
      sp.gate = nullptr;
      if (fold) {
        sp.row_ssq = P->row_stats;
        sp.ssq_ld = T;
      }
      rc = skinny_gemm_run(SK_EPI_GATED_RESID, sp, L.w_down, L.w_down, W, W, act, F, 0, stream);
      if (rc) break;
    }
  }
  return rc;
}

}  // extern "C"
