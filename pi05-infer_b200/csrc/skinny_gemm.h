// Internal interface of the swap-AB tcgen05 GEMM (see skinny_gemm.cu).
#pragma once

#include <cuda_bf16.h>
#include <stddef.h>

namespace pi05 {

enum SkinnyEpi : int {
  SK_EPI_STORE = 0,        // out[t, n] = act(bf16(y + bias[n] + pos[t % pos_rows, n]))   (bias, pos, act optional)
  SK_EPI_GATED_RESID = 1,  // out[t, n] = bf16(resid[t, n] + bf16(y + bias[n]) * bf16(gate[n]))   (bias, gate optional)
  SK_EPI_GEGLU = 2,        // out[t, n] = bf16(gelu_tanh(bf16(y_gate)) * y_up)
  SK_EPI_QKV_ROPE = 3,     // RoPE(q) -> q_out, RoPE(k) / v -> KV cache rows krow0 + t
};

struct SkinnyParams {
  int m_tok = 0;     // valid tokens
  int k = 0;         // reduction length (multiple of 8; a ragged last 64-block is zero-filled)
  int n_tiles = 0;   // 128-row weight tiles
  int kb_total = 0;  // set by the launcher
  int splits = 1;    // set by the launcher
  int cluster = 0;   // set by the launcher: 1 = the splits of a tile form a cluster and reduce through DSMEM
  int allow_cluster = 1;  // 0 = split-K only through the global accumulator
  int allow_wide = 1;     // 0 = stay on this kernel for more than 128 tokens (token tiles on blockIdx.y)
  int max_tok = 0;        // 64 = 64-token tiles whatever the token count (0 = 64 / 128 / 256 by count)
  int push = 0;      // set by the launcher: cluster split-K pushes partial slices to their owners (TOK 64)
  // STORE / GATED_RESID / GEGLU
  __nv_bfloat16* out = nullptr;
  int ldo = 0;
  const __nv_bfloat16* resid = nullptr;
  int ldr = 0;
  const float* gate = nullptr;
  const float* bias = nullptr;   // fp32 [n]
  const float* pos = nullptr;    // fp32 [pos_rows, n] added before rounding (patch embedding)
  int pos_rows = 0;
  int act = 0;                   // 0 none, 1 gelu_tanh on the bf16-rounded value
  int n_valid = 0;               // output columns (multiple of 8); 0 = n_tiles * 128
  // QKV_ROPE
  const __nv_bfloat16* cos = nullptr;  // [m_tok, head_dim]
  const __nv_bfloat16* sin = nullptr;
  __nv_bfloat16* q_out = nullptr;      // [m_tok, n_q_heads, head_dim]
  __nv_bfloat16* k_cache = nullptr;    // [n_kv_heads][kv_rows][head_dim]
  __nv_bfloat16* v_cache = nullptr;
  size_t kv_head_stride = 0;           // elements between KV heads
  int krow0 = 0;
  int n_q_heads = 0;
  int n_kv_heads = 0;
  int head_dim = 0;
  // Row statistics for a following RMS norm (STORE / GATED_RESID): when set, the
  // sum of squares of every token's bf16 outputs within each part of the output
  // columns is written to row_ssq[part * ssq_ld + token] (fixed summation order).
  // A part is a 128-row weight tile in the small-token kernel and a 64-column slab
  // in the many-token one; row_ssq_parts() gives the count for a launch.
  float* row_ssq = nullptr;
  int ssq_ld = 0;
  float* row_sum = nullptr;  // many-token kernel: the parts' plain sums, same layout (LayerNorm means)
  // Folded (ada)RMS norm of the X operand (GEGLU / QKV_ROPE): X holds
  // the raw residual stream h and the weights carry the norm's (1 + scale) in their
  // columns (pi05_fold_adarms), so the norm reduces to a per-token factor and a
  // per-row bias applied to the accumulator before the epilogue:
  //   y[r, t] = acc[r, t] * rstd[t] + bias(r)      (bias added by split 0 only)
  //   rstd[t] = rsqrt(sum_j fold_ssq[j * fold_ld + t] / fold_d + fold_eps)
  // over fold_parts partial sums in order; bias(r) = fold_bias0[weight row] for the
  // rows of map 0 and fold_bias1[weight row] for those of map 1 (W . shift, fp32).
  // The small-token kernel (<= 64 tokens) needs both bias vectors; the many-token
  // kernel applies rstd only (plain RMSNorm: its (1 + w) lives in the weights) and
  // takes no bias.
  const float* fold_ssq = nullptr;
  int fold_parts = 0;
  int fold_ld = 0;
  int fold_d = 0;
  float fold_eps = 0.f;
  const float* fold_bias0 = nullptr;
  const float* fold_bias1 = nullptr;
  // Folded LayerNorm (STORE, many-token kernel): with ln_sum set (per-part sums of x
  // in fold_ssq's layout) the weights carry the LayerNorm's gamma, `bias` holds
  // b + W . beta, and ln_colsum[n] = sum_k W'[n, k] of the folded bf16 weights; the
  // accumulator becomes  y = rstd[t] * (acc - mean[t] * ln_colsum[n]) + bias[n]  with
  // mean = sum / fold_d, rstd = rsqrt(ssq / fold_d - mean^2 + fold_eps).
  const float* ln_sum = nullptr;
  const float* ln_colsum = nullptr;
  // Optional timing trace: word 0 is a slot counter, word 1 the capacity in
  // records (records beyond it are dropped); each CTA appends 8 words at 8 + 8*slot
  // {tag << 32 | cta, entry, after prologue, after grid-dependency wait,
  //  accumulator ready, partial published (global split-K), epilogue done,
  //  first weight TMA issued}.
  unsigned long long* trace = nullptr;
  int trace_tag = 0;
  // Failure-path test hook (global split-K path only; set by the launcher from
  // pi05_debug_set_fault): split fault_skip_split of tile 0 neither publishes nor
  // arrives, and the arrival wait gives up after wait_ns (0 = kWaitTimeoutNs).
  int fault_skip_split = -1;
  unsigned long long wait_ns = 0;
  // workspace
  float* accum = nullptr;   // fp32 split-K accumulator (zero on entry, left zero on exit)
  size_t accum_bytes = 0;
  int* counters = nullptr;  // split-K tickets (zero on entry, left zero on exit)
  int* status = nullptr;    // device status word
};

constexpr int kNormMaxParts = 16;  // folded-norm partial sums of squares per token

// Parts per token that a GATED_RESID / STORE launch of m_tok tokens and n_cols
// output columns writes to row_ssq (the kernel it will run on decides).
int row_ssq_parts(int m_tok, int n_cols);
int skinny_choose_splits(int n_tiles, int kb_total, int tok_tiles, int sms);
int skinny_choose_splits_cluster(int n_tiles, int kb_total, int tok_tiles, int sms, int max_cluster);

// w0/w1: weight matrices for the two 64-row boxes of each tile (the same matrix
// except for GEGLU, where w0 = gate and w1 = up).  w_rows*: their row counts.
int skinny_gemm_run(int epi, SkinnyParams p, const void* w0, const void* w1, int w_rows0, int w_rows1,
                    const void* x, int ldx, int splits_override, void* stream);

}  // namespace pi05
