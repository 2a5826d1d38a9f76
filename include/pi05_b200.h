/*
 * pi05_b200 — C ABI of the B200 (sm_100a) kernels behind pi0.5 sample_actions.
 *
 * Conventions
 *  - Every pointer is a device pointer unless named host_*; tensors are dense
 *    row-major; bf16 tensors are passed as void*, fp32 as float*.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Nothing here allocates or frees device memory.  Ops that need scratch take a
 *    caller-owned `workspace` of pi05_workspace_bytes() bytes, 256-byte aligned,
 *    zero-filled once before first use.  Its first 16 KiB (status word and
 *    split-K barrier counters) must not be modified by the caller; every op
 *    leaves the counters at zero.  The rest is scratch.  Ops that share one
 *    workspace must be ordered on one stream.
 *  - Return value: 0 on success, else a PI05_ERR_* code (pi05_status.h);
 *    pi05_last_error() gives a one-line reason.  No C++ exception crosses the ABI.
 *  - Kernels give up any internal wait after 2 s and OR a PI05_DEV_* bit into the
 *    workspace status word instead of hanging; pi05_read_device_status() reads it.
 *
 * Each entry point names the reference interface it replaces (paths inside the
 * chenchaoxu7575/pi05-infer tree).
 */
#ifndef PI05_B200_H
#define PI05_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- library ----------------------------------------------------------- */

/* ABI version (bumped on any signature change). */
int pi05_abi_version(void);

/* Text of the last error on this host thread ("" if none). */
const char* pi05_last_error(void);

/* Workspace bytes needed by the ops below for up to `max_tokens` activation rows
 * (tokens x batch) and attention over up to `max_kv` keys. */
size_t pi05_workspace_bytes(int max_tokens, int max_kv);

/* Synchronise `stream`, copy the workspace status word to *host_status and clear
 * it.  Returns PI05_ERR_DEVICE if the word was non-zero; in that case the
 * workspace's split-K counters are also reset, so that the next call starts from
 * a clean state after a kernel gave up on a wait. */
int pi05_read_device_status(void* workspace, int* host_status, void* stream);

/* Number of kernel launches this library has issued in this process (a CUDA-graph
 * capture counts the launches it records). */
long long pi05_launch_count(void);

/* Test hook for the split-K path: force the split count of the skinny GEMMs
 * (0 = automatic).  Process-wide. */
void pi05_debug_set_splits(int splits);

/* Profiling hook: device buffer that the GEMM ops called through this header
 * append per-CTA timestamp records to (word 0: record counter, word 1: capacity
 * in records; record i at words 8 + 8 i).  NULL disables.  Process-wide. */
void pi05_debug_set_trace(unsigned long long* buf);

/* Failure-path test hook -- no counterpart in the reference.  While armed
 * (skip_split >= 0), the split-K GEMMs run their global-memory split-K path, in
 * which split `skip_split` of the first output tile neither publishes its
 * partial nor arrives at the tile's counter, and the arrival wait gives up after
 * wait_ns nanoseconds (0 = the built-in 2 s limit).  The waiting CTAs then set
 * PI05_DEV_TIMEOUT_EPILOGUE in the device status word, skip the tile's epilogue
 * and exit normally, so the context stays usable.  skip_split < 0 disarms.
 * Process-wide; for tests only. */
void pi05_debug_set_fault(int skip_split, unsigned long long wait_ns);

/* ---- fused denoise ops (swap-AB tcgen05 GEMM + fused epilogue) ---------- */

/* out[m, n] = gelu_tanh(bf16(x @ wg^T)) * (x @ wu^T), bf16.
 * Replaces torch.ops.pi05_infer.gate_up_geglu
 * (pi05_infer/gemma/rlinf_fused_denoise.py:350-389).
 * x [m, k], wg/wu [n, k]; k % 64 == 0, n % 64 == 0. */
int pi05_gate_up_geglu(const void* x, const void* wg, const void* wu, void* out, int m, int n, int k,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Fused q|k|v projection + RoPE + static-KV tail write.
 * Replaces torch.ops.pi05_infer.qkv_rope_kv (rlinf_fused_denoise.py:392-467).
 * x [m, k]; w [(hq + 2*hkv) * d, k] = cat(q_proj, k_proj, v_proj) rows;
 * cos/sin [m, d] bf16; q_out [m, hq, d]; k_cache/v_cache [hkv, kv_rows, d]
 * receive rows krow0 .. krow0+m-1.  d % 128 == 0, k % 64 == 0. */
int pi05_qkv_rope_kv(const void* x, const void* w, const void* cos, const void* sin, void* q_out, void* k_cache,
                     void* v_cache, int m, int k, int krow0, int kv_rows, int n_q_heads, int n_kv_heads,
                     int head_dim, void* workspace, size_t workspace_bytes, void* stream);

/* pi05_gate_up_geglu for callers that cannot allocate device memory -- no
 * counterpart in the reference.  Same math and arguments minus the workspace:
 * the split-K scratch is a fixed 4 MiB (+4 KiB) device array inside this library,
 * held by every GPU that loads it until the process exits.  Limits: m <= 64,
 * n <= 16384, k <= 16384 (n % 64 == 0, k % 64 == 0); larger shapes return
 * PI05_ERR_SHAPE.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress), so make that call before any stream capture.  All calls
 * share the one array: calls that can overlap on the GPU (different streams,
 * different host threads on one device) race and must be serialised by the caller. */
int pi05_gate_up_geglu_noalloc(const void* x, const void* wg, const void* wu, void* out, int m, int n, int k,
                               void* stream);

/* Status of pi05_gate_up_geglu_noalloc on the current device -- no counterpart in
 * the reference.  Synchronises `stream`, copies the built-in scratch's status word
 * (nonzero = a kernel wait timed out and its output is not valid) to *host_status,
 * clears it, and returns PI05_ERR_DEVICE when it was nonzero.  The word is sticky:
 * calls of the entry point do not clear it, so a timeout of any earlier call is
 * reported by the next read.  Allocates nothing. */
int pi05_gate_up_geglu_noalloc_status(int* host_status, void* stream);

/* out[m, n] = bf16(resid[m, n] + bf16(x @ w^T) * bf16(gate[n])); gate NULL -> plain residual.
 * Replaces o_proj / down_proj + _gated_residual
 * (pi05_infer/gemma/modeling_gemma.py:455-456, 138-148, 231-249).
 * out may alias resid.  n % 128 == 0, k % 64 == 0. */
int pi05_linear_gated_residual(const void* x, const void* w, const void* resid, const float* gate, void* out,
                               int m, int n, int k, void* workspace, size_t workspace_bytes, void* stream);

/* out[m, n] = bf16(x @ w^T) (nn.Linear without bias, bf16).  n % 128 == 0, k % 64 == 0. */
int pi05_linear(const void* x, const void* w, void* out, int m, int n, int k, void* workspace,
                size_t workspace_bytes, void* stream);


/* ---- normalisation, attention, glue ------------------------------------- */

/* adaRMSNorm (mod != NULL, mod = [scale | shift | gate] fp32 [3*d]) or Gemma RMSNorm
 * (mod == NULL, weight fp32 [d], scale (1 + weight)); fp32 statistics, bf16 out.
 * Replaces GemmaRMSNorm.forward (pi05_infer/gemma/modeling_gemma.py:65-116).
 * x, out [rows, d] with row pitches ldx / ldo (elements); d % 8 == 0. */
int pi05_rms_norm(const void* x, int ldx, const float* mod, const float* weight, void* out, int ldo, int rows, int d,
                  float eps, void* stream);

/* Multi-query attention, one KV head shared by all query heads.
 * Replaces eager_attention_forward + repeat_kv (modeling_gemma.py:219-228, 252-275).
 * q [rows, head_dim] (row = token * n_heads + head), k/v [kv_len, head_dim],
 * key_valid [kv_len] bytes (0 = masked key), out [rows, head_dim].
 * head_dim == 256.  splits <= 0 picks the split-KV factor automatically. */
int pi05_attention(const void* q, const void* k, const void* v, const uint8_t* key_valid, void* out, int rows,
                   int kv_len, int head_dim, float scale, int splits, void* workspace, size_t workspace_bytes,
                   void* stream);

/* h[rows, dout] = bf16(x @ w^T + b), fp32 math.  Replaces action_in_proj
 * (pi05_infer/openpi_patched/pi0_pytorch.py:303-323).  din <= 64. */
int pi05_action_in(const float* x, const float* w, const float* b, void* h, int rows, int din, int dout,
                   void* stream);

/* Final adaRMSNorm -> fp32 -> action_out_proj -> flow_ode Euler update of x_t in
 * place (modeling_gemma.py:782-783; engine.py:664-675, 754-767).  v_out (may be
 * NULL) receives the velocity.  d a multiple of 256 up to 2048, h / w / mod
 * 16-byte aligned, dout <= 64. */
int pi05_final_euler(const void* h, const float* mod, const float* w, const float* b, float* x_t, float* v_out,
                     int rows, int d, int dout, float eps, float t, float delta, void* stream);

/* RoPE cos/sin tables [rows, d] bf16 from a key-validity mask (GemmaRotaryEmbedding,
 * modeling_gemma.py:151-182).  mode 0: prefix rows, position = cumsum(valid) - 1
 * (engine.py:778); mode 1: suffix rows, position = sum(valid[0:n_prefix]) + row
 * (engine.py:476-477).  inv_freq [d/2] fp32.  n_prefix <= 4096. */
int pi05_rope_table(const uint8_t* valid, int n_prefix, int mode, int rows, const float* inv_freq, int d, void* cos,
                    void* sin, void* stream);

/* adaRMS modulation table for every denoise step (engine.py:556-599):
 * table[s] = stack_i(dense_i(silu(time_mlp_out(silu(time_mlp_in(sinusoid(t_s))))))),
 * all fp32.  timesteps [n_steps] device fp32; w_dense [n_norm*3*width, width] and
 * b_dense [n_norm*3*width] are the norms' dense layers stacked in forward order;
 * table [n_steps, n_norm*3*width].  n_steps <= 16. */
int pi05_adarms_table(const float* timesteps, int n_steps, int width, const float* w_tin, const float* b_tin,
                      const float* w_tout, const float* b_tout, const float* w_dense, const float* b_dense,
                      int n_norm, float* table, void* workspace, size_t workspace_bytes, void* stream);

/* ---- whole denoise loop --------------------------------------------------- */

/* Per-layer device pointers of the action expert (bf16 weights, reference layout). */
typedef struct Pi05ExpertLayer {
  const void* w_qkv;   /* [(hq + 2*hkv) * d, width]: cat(q_proj, k_proj, v_proj) */
  const void* w_o;     /* [width, hq * d] */
  const void* w_gate;  /* [mlp, width] */
  const void* w_up;    /* [mlp, width] */
  const void* w_down;  /* [width, mlp] */
  void* k_cache;       /* [hkv, kv_rows, d]; rows [0, prefix_len) hold the prefix keys */
  void* v_cache;
} Pi05ExpertLayer;

/* Per-(step, layer) folded projections for the folded-norm denoise path (see
 * pi05_fold_adarms): the layer's q|k|v and gate/up weights with that step's
 * input_layernorm / post_attention_layernorm (1 + scale) folded into their columns,
 * and the matching fp32 biases W . shift. */
typedef struct Pi05ExpertFold {
  const void* w_qkv;    /* [(hq + 2*hkv) * d, width] bf16 */
  const void* w_gate;   /* [mlp, width] bf16 */
  const void* w_up;     /* [mlp, width] bf16 */
  const float* b_qkv;   /* [(hq + 2*hkv) * d] */
  const float* b_gate;  /* [mlp] */
  const float* b_up;    /* [mlp] */
} Pi05ExpertFold;

/* Everything one denoise step touches.  Host memory owned by the caller. */
typedef struct Pi05ExpertPlan {
  int depth, width, mlp_dim, n_q_heads, n_kv_heads, head_dim;
  int tokens;              /* action horizon (50) */
  int action_dim;          /* 32 */
  int prefix_len;          /* rows of the KV cache holding prefix keys (P) */
  int kv_rows;             /* >= prefix_len + tokens */
  float eps;
  const Pi05ExpertLayer* layers;  /* host array [depth] */
  int num_steps;
  const float* host_timesteps;    /* host [num_steps + 1]: 1, ..., 1/N, 0 */
  const float* mod_table;         /* [num_steps, 2*depth+1, 3*width] fp32 */
  const float* w_in;              /* action_in_proj [width, action_dim] fp32 */
  const float* b_in;
  const float* w_out;             /* action_out_proj [action_dim, width] fp32 */
  const float* b_out;
  const void* rope_cos;           /* [tokens, d] bf16 */
  const void* rope_sin;
  const uint8_t* key_valid;       /* [prefix_len + tokens] */
  float* x_t;                     /* [tokens, action_dim] fp32: noise in, actions out */
  float* v_t;                     /* [tokens, action_dim] fp32: last velocity (may be NULL) */
  void* h;                        /* [tokens, width] bf16 residual stream */
  void* xn;                       /* [tokens, width] bf16 normalised input */
  void* q;                        /* [tokens, hq, d] bf16 */
  void* attn;                     /* [tokens, hq * d] bf16 */
  void* act;                      /* [tokens, mlp] bf16 */
  void* workspace;
  size_t workspace_bytes;
  int attn_splits;                /* <= 0: automatic */
  unsigned long long* trace;      /* optional device buffer for per-CTA timestamp records of the
                                     loop's GEMM and attention launches (layout of pi05_debug_set_trace),
                                     NULL = off */
  const Pi05ExpertFold* fold;     /* host array [num_steps * depth] (step-major), or NULL.  When set,
                                     pi05_denoise_step runs no norm kernel inside
                                     the layers: q|k|v and gate/up read the residual stream h with these
                                     folded weights and scale each token by its rstd from the row
                                     statistics that action_in / o_proj / down_proj write. */
  int batch;                      /* independent observations denoised together (0 or 1: one).  With
                                     batch = B > 1 every GEMM runs over B * tokens rows (observation b's
                                     rows b * tokens ..); x_t, v_t, h, xn, q, attn, act, rope_cos and
                                     rope_sin hold B * tokens rows; each layer's k_cache / v_cache hold
                                     B caches [hkv, kv_rows, d] back to back and key_valid B masks of
                                     kv_rows; kv_stage is needed. */
  void* kv_stage;                 /* batch > 1: [2][B * tokens][d] bf16 staging of the new K / V rows */
  const float* host_step_coefs;   /* host [num_steps][3] or NULL (flow_ode): the sampler's update
                                     x <- (x - v t) * c0 + (x + v (1 - t)) * c1 + c2 * noise, as
                                     sample_mean_var_val computes mean and std for flow_sde / flow_cps
                                     (_extract_src/openpi_action_model.py:984-1006) */
  const float* step_noise;        /* [num_steps][B * tokens][action_dim] fp32 N(0, 1), read where
                                     c2 != 0 */
} Pi05ExpertPlan;

/* Folds an adaRMS norm into the projection that consumes its output, for the
 * folded-norm denoise path (Pi05ExpertFold).  The reference normalises first and
 * projects the bf16 result (GemmaRMSNorm adaRMS, modeling_gemma.py:82-116, then
 * the q|k|v or gate/up projection); with
 *   w_out[n, j] = bf16(w[n, j] * (1 + scale[j])),   b_out[n] = sum_j w[n, j] * shift[j] (fp32)
 * that projection becomes rstd[t] * (w_out . h[t]) + b_out.  w, w_out [rows, k]
 * bf16 (16-byte aligned, k % 8 == 0); scale, shift [k] fp32; b_out [rows] fp32. */
int pi05_fold_adarms(const void* w, int rows, int k, const float* scale, const float* shift, void* w_out,
                     float* b_out, void* stream);

/* One Euler step `step` (0-based) of the denoise loop: action_in_proj, 18 expert
 * layers, final norm, action_out_proj, Euler update of plan->x_t.
 * Replaces one replay of the reference's captured step (engine.py:629-676, 908-1001). */
int pi05_denoise_step(const Pi05ExpertPlan* plan, int step, void* stream);

/* All plan->num_steps steps (engine.py:390-405), one launch per kernel phase. */
int pi05_denoise_loop(const Pi05ExpertPlan* plan, void* stream);



/* ---- prefix (PaliGemma Gemma-2B over image + language tokens) ------------- */

/* out[i, :] = bf16(bf16(table[ids[i], :]) * scale): embed_tokens(ids) * sqrt(width)
 * (pi05_infer/openpi_patched/pi0_pytorch.py:225-228).  ids int32, table bf16 [vocab, d],
 * out row pitch ldo; d % 8 == 0.  Out-of-range ids produce a zero row and set
 * PI05_DEV_BAD_INDEX in the workspace status word. */
int pi05_embed_tokens(const void* table, int vocab, const int32_t* ids, int n, int d, float scale, void* out,
                      int ldo, void* workspace, size_t workspace_bytes, void* stream);

typedef struct Pi05PrefixLayer {
  const void* w_qkv;    /* [(hq + 2*hkv) * d, width] = cat(q_proj, k_proj, v_proj) (prefix_qkv_fused.py:132-139) */
  const void* w_o;      /* [width, hq * d] */
  const void* w_gate;   /* [mlp, width] */
  const void* w_up;
  const void* w_down;   /* [width, mlp] */
  const float* ln1_w;   /* input_layernorm weight fp32 [width] (scale 1 + w) */
  const float* ln2_w;   /* post_attention_layernorm weight fp32 [width] */
  void* k_cache;        /* [hkv, kv_rows, d]: rows [0, tokens) receive this layer's prefix K */
  void* v_cache;
  /* Folded copies for the folded-norm path, or NULL (then the norm kernels run):
   * w_qkv with (1 + ln1_w) and w_gate / w_up with (1 + ln2_w) folded into their
   * columns (pi05_fold_adarms with a zero shift). */
  const void* wf_qkv;
  const void* wf_gate;
  const void* wf_up;
} Pi05PrefixLayer;

typedef struct Pi05PrefixPlan {
  int depth, width, mlp_dim, n_q_heads, n_kv_heads, head_dim;
  int tokens;                    /* prefix length P (<= 4096) */
  int kv_rows;                   /* >= tokens */
  float eps;
  const Pi05PrefixLayer* layers; /* host array [depth] */
  const uint8_t* key_valid;      /* [tokens] pad mask (1 = real token) */
  const float* inv_freq;         /* [d/2] fp32 */
  void* rope_cos;                /* [tokens, d] bf16 scratch */
  void* rope_sin;
  void* h;                       /* [tokens, width] bf16: prefix embeddings in; residual stream */
  void* xn;                      /* [tokens, width] bf16 */
  void* q;                       /* [tokens, hq, d] bf16 */
  void* attn;                    /* [tokens, hq * d] bf16 */
  void* act;                     /* [tokens, mlp] bf16 */
  void* workspace;
  size_t workspace_bytes;
  int kv_only_last_layer;        /* 1: the last layer stops after K/V (prefix_last_layer.py:46-112) */
  float* row_stats;              /* [width / 64, tokens] fp32 scratch for the folded norms, or NULL.  With
                                    it and every layer's wf_* set, no norm kernel runs: the residual
                                    GEMMs write per-64-column sums of squares of h, and q|k|v and
                                    gate/up scale their accumulators by each token's rstd. */
} Pi05PrefixPlan;

/* Prefix LM forward with use_cache=True: fills every layer's K/V cache rows
 * [0, tokens).  Replaces PaliGemmaWithExpertModel.forward(inputs_embeds=[prefix, None])
 * (gemma_pytorch.py:131-142) as called by _build_prefix_cache (engine.py:770-794). */
int pi05_prefix_forward(const Pi05PrefixPlan* plan, void* stream);


/* ---- SigLIP So400m/14 vision tower + projector ---------------------------- */

/* LayerNorm (fp32 statistics, fp32 weight/bias), bf16 in/out; x row pitch d.
 * Replaces the SigLIP layer_norm1 / layer_norm2 / post_layernorm modules. */
int pi05_layer_norm(const void* x, const float* w, const float* b, void* out, int ldo, int rows, int d, float eps,
                    void* stream);

/* Per-head attention of the SigLIP encoder: qkv [views*seq, 3*width] (q | k | v,
 * head h at columns h*head_dim of each), out [views*seq, width]; no mask,
 * scale head_dim^-0.5.  head_dim == 72, seq == 256. */
int pi05_siglip_attention(const void* qkv, int views, int seq, int width, int heads, int head_dim, void* out,
                          void* stream);

typedef struct Pi05SiglipLayer {
  const void* w_qkv;   /* [3*width, width] bf16 = cat(q_proj, k_proj, v_proj) */
  const float* b_qkv;  /* [3*width] */
  const void* w_o;     /* out_proj [width, width] */
  const float* b_o;
  const void* w_fc1;   /* [mlp, width] */
  const float* b_fc1;
  const void* w_fc2;   /* [width, mlp] */
  const float* b_fc2;
  const float* ln1_w;
  const float* ln1_b;
  const float* ln2_w;
  const float* ln2_b;
  /* Folded LayerNorms, or NULL (then the LayerNorm kernels run): q|k|v and fc1 with
   * the preceding LayerNorm's gamma folded into their columns (bf16), their biases
   * b + W . beta (fp32), and the column sums sum_k W'[n, k] of the folded weights. */
  const void* wf_qkv;
  const float* bf_qkv;
  const float* cs_qkv;
  const void* wf_fc1;
  const float* bf_fc1;
  const float* cs_fc1;
} Pi05SiglipLayer;

typedef struct Pi05SiglipPlan {
  int depth, width, mlp_dim, n_heads, head_dim, patch, image_size, num_views, proj_dim;
  float eps;
  const Pi05SiglipLayer* layers;  /* host array [depth] */
  const void* w_patch;            /* [width, k_pad] bf16: conv weight flattened (c, ky, kx), zero-padded */
  const float* b_patch;           /* [width] */
  const float* pos_emb;           /* [patches, width] fp32 */
  int k_pad;                      /* >= 3*patch*patch, multiple of 64 */
  const float* post_ln_w;
  const float* post_ln_b;
  const void* w_proj;             /* multi_modal_projector [proj_dim, width] bf16 */
  const float* b_proj;
  const float* images;            /* [views, 3, image_size, image_size] fp32 in [-1, 1] */
  void* cols;                     /* [views*patches, k_pad] bf16 scratch */
  void* h;                        /* [views*patches, width] bf16 */
  void* xn;                       /* [views*patches, width] bf16 */
  void* qkv;                      /* [views*patches, 3*width] bf16 */
  void* attn;                     /* [views*patches, width] bf16 */
  void* act;                      /* [views*patches, mlp] bf16 */
  void* out;                      /* [views*patches, proj_dim] bf16 (rows of the prefix buffer) */
  int ldo;
  void* workspace;
  size_t workspace_bytes;
  const void* wf_proj;            /* projector with post_layernorm folded in, or NULL */
  const float* bf_proj;
  const float* cs_proj;
  float* row_stats;               /* [2][width / 64][views*patches] fp32 (sums, sums of squares), or NULL.
                                     With it and every wf_* set, no LayerNorm kernel runs: the residual
                                     GEMMs and the patch embedding write per-64-column statistics of h,
                                     and q|k|v, fc1 and the projector normalise in their epilogues. */
} Pi05SiglipPlan;

/* All views through SigLIP and the projector into `out`.  Replaces embed_image /
 * PaliGemma get_image_features (gemma_pytorch.py:106-107) over cat(images)
 * (pi0_pytorch.py:203-217). */
int pi05_siglip_forward(const Pi05SiglipPlan* plan, void* stream);

/* ---- observation preprocessing and action output transform ---------------- */

/* Camera images as the environment gives them, uint8 [n, h, w, 3] (layout 0) or
 * [n, 3, h, w] (layout 1), to the model's fp32 [n, 3, size, size] in [-1, 1]:
 * p / 255 * 2 - 1 after a bilinear resize (half-pixel centres) that keeps the
 * aspect ratio and fits the longer side, the border filled with -1.  An image
 * already size x size is copied pixel for pixel.  Replaces the image part of
 * openpi's preprocess_observation_pytorch (called at pi0_pytorch.py:165-174) and of
 * the input transforms that predict_action_batch runs (engine.py:321-342). */
int pi05_preprocess_images(const uint8_t* images, int n, int h, int w, int layout, float* out, int size,
                           void* stream);

/* out[r, j] = normalised x[r, j] for j < din (statistics for j < nstat, the rest
 * passed through), 0 for din <= j < dout.  mode 0: (x - a) / (b + 1e-6) with
 * a = mean, b = std; mode 1: (x - a) / (b - a + 1e-6) * 2 - 1 with a = q01,
 * b = q99.  Replaces openpi Normalize + PadStatesAndActions on the state
 * (input transforms built at builder.py:120-128). */
int pi05_normalize_rows(const float* x, int rows, int din, const float* a, const float* b, int nstat, int mode,
                        float* out, int dout, void* stream);

/* out[r, j] = un-normalised x[r, j] for j < dout <= din: mode 0: x * (b + 1e-6) + a;
 * mode 1: (x + 1) / 2 * (b - a + 1e-6) + a; statistics for j < nstat.  Replaces
 * openpi Unnormalize on the actions and the policy's output slice (builder.py:129-136,
 * dataconfig/policies/turtle_policy.py:89-93, libero_policy.py LiberoOutputs). */
int pi05_unnormalize_rows(const float* x, int rows, int din, const float* a, const float* b, int nstat, int mode,
                          float* out, int dout, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PI05_B200_H */
