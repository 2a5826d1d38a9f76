// SigLIP So400m/14 vision tower + PaliGemma projector (embed_image,
// pi05_infer/openpi_patched/gemma_pytorch.py:106-107; all views batched as in
// pi0_pytorch.py:203-217).
//
//   cols  = im2col(images)                          14x14 patches, (c, ky, kx) order, K padded to 64
//   h     = bf16(cols @ Wpatch^T + b + pos)         patch conv + position embedding
//   27 x: h += out_proj(MHA(LN1(h)))                q|k|v fused, bias
//         h += fc2(gelu_tanh(fc1(LN2(h))))
//   out   = LN_post(h) @ Wproj^T + b                written into the prefix buffer
//
// The GEMMs use the swap-AB tcgen05 kernel (bias / GELU / residual epilogues).
// Attention is per head (16 heads x 72 dims, 256 tokens per view, no mask), a
// tcgen05 kernel over whole rows (siglip_attn_tc.cu).
#include <cmath>
#include <cstdlib>

#include "../../include/pi05_b200.h"
#include "elementwise.h"
#include "host_util.h"
#include "ptx.cuh"
#include "skinny_gemm.h"

using namespace pi05;

namespace {

// LayerNorm over the last dim: fp32 mean/variance, y = (x - mean) * rstd * w + b, bf16 out.
__global__ void __launch_bounds__(128) layer_norm_kernel(const __nv_bfloat16* __restrict__ x,
                                                         const float* __restrict__ w, const float* __restrict__ b,
                                                         __nv_bfloat16* __restrict__ out, int ldo, int d, float eps) {
  __shared__ float red[4];
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int row = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const __nv_bfloat16* xr = x + (size_t)row * d;
  float s = 0.f;
  for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += __bfloat162float(v[j]);
  }
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  const float mean = (red[0] + red[1] + red[2] + red[3]) / (float)d;
  __syncthreads();
  float q = 0.f;
  for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float c = __bfloat162float(v[j]) - mean;
      q += c * c;
    }
  }
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffff, q, o);
  if (lane == 0) red[warp] = q;
  __syncthreads();
  const float rstd = rsqrtf((red[0] + red[1] + red[2] + red[3]) / (float)d + eps);
  for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(&u);
    __align__(16) __nv_bfloat16 o8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o8[j] = __float2bfloat16((__bfloat162float(v[j]) - mean) * rstd * w[i + j] + b[i + j]);
    *reinterpret_cast<uint4*>(out + (size_t)row * ldo + i) = *reinterpret_cast<const uint4*>(o8);
  }
}

// im2col for the 14x14/14 patch conv: cols[v*gp*gp + py*gp + px, c*P*P + ky*P + kx] =
// bf16(img[v, c, py*P + ky, px*P + kx]); columns [3*P*P, k_pad) are zero.
__global__ void __launch_bounds__(256) im2col_kernel(const float* __restrict__ img, int views, int hw, int patch,
                                                     int k_pad, __nv_bfloat16* __restrict__ cols) {
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int gp = hw / patch;
  const int kk = 3 * patch * patch;
  const size_t total = (size_t)views * gp * gp * k_pad;
  for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (size_t)gridDim.x * blockDim.x) {
    const int k = (int)(idx % k_pad);
    const size_t row = idx / k_pad;
    float val = 0.f;
    if (k < kk) {
      const int v = (int)(row / (gp * gp)), pidx = (int)(row % (gp * gp));
      const int py = pidx / gp, px = pidx % gp;
      const int c = k / (patch * patch), r = k % (patch * patch);
      const int ky = r / patch, kx = r % patch;
      val = img[(((size_t)v * 3 + c) * hw + (py * patch + ky)) * hw + px * patch + kx];
    }
    cols[idx] = __float2bfloat16(val);
  }
}

constexpr int kHd = 72;  // SigLIP head dim

inline bool nz(const void* p) { return p != nullptr; }

}  // namespace

namespace pi05 {
// The attention kernel (tcgen05, siglip_attn_tc.cu).
int siglip_attention_tc_run(const void* qkv, int views, int width, int heads, void* out, int* status,
                            cudaStream_t stream);
}  // namespace pi05

namespace {

int siglip_attention_run(const void* qkv, int views, int seq, int width, int heads, int head_dim, void* out,
                         void* stream, int* status = nullptr) {
  if (!nz(qkv) || !nz(out)) {
    set_last_error("siglip_attention: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (head_dim != kHd || seq != 256 || heads * head_dim != width || views <= 0 || !aligned16(qkv) ||
      !aligned16(out)) {
    set_last_error("siglip_attention: supports head_dim 72, 256 tokens per view, 16-byte aligned buffers");
    return PI05_ERR_SHAPE;
  }
  return siglip_attention_tc_run(qkv, views, width, heads, out, status, reinterpret_cast<cudaStream_t>(stream));
}

// PI05_FOLD_NORM=0 in the environment keeps the LayerNorm kernels.
bool siglip_fold_enabled() {
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

int pi05_layer_norm(const void* x, const float* w, const float* b, void* out, int ldo, int rows, int d, float eps,
                    void* stream) {
  if (!nz(x) || !nz(w) || !nz(b) || !nz(out)) {
    set_last_error("layer_norm: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (rows <= 0 || d % 8 || ldo % 8 || !aligned16(x) || !aligned16(out)) {
    set_last_error("layer_norm: need d, ldo multiples of 8 and 16-byte aligned x/out");
    return PI05_ERR_SHAPE;
  }
  return launch_pdl(layer_norm_kernel, dim3(rows), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream),
                    pdl_enabled(), static_cast<const __nv_bfloat16*>(x), w, b, static_cast<__nv_bfloat16*>(out), ldo,
                    d, eps);
}

int pi05_siglip_attention(const void* qkv, int views, int seq, int width, int heads, int head_dim, void* out,
                          void* stream) {
  return siglip_attention_run(qkv, views, seq, width, heads, head_dim, out, stream);
}

int pi05_siglip_forward(const Pi05SiglipPlan* P, void* stream) {
  if (!nz(P) || !nz(P->layers) || !nz(P->images) || !nz(P->w_patch) || !nz(P->out)) {
    set_last_error("siglip_forward: null plan field");
    return PI05_ERR_INVALID_ARG;
  }
  const int W = P->width, F = P->mlp_dim, V = P->num_views;
  const int gp = P->image_size / P->patch, S = gp * gp, T = V * S;
  if (W % 128 || F % 8 || P->k_pad % 64 || P->k_pad < 3 * P->patch * P->patch || S != 256 ||
      P->n_heads * P->head_dim != W || P->proj_dim % 128) {
    set_last_error("siglip_forward: unsupported shape");
    return PI05_ERR_SHAPE;
  }
  Workspace ws;
  if (split_workspace(P->workspace, P->workspace_bytes, &ws)) {
    set_last_error("siglip_forward: workspace missing or too small");
    return PI05_ERR_WORKSPACE;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  auto* h = static_cast<__nv_bfloat16*>(P->h);
  auto* xn = static_cast<__nv_bfloat16*>(P->xn);
  auto* qkv = static_cast<__nv_bfloat16*>(P->qkv);
  auto* attn = static_cast<__nv_bfloat16*>(P->attn);
  auto* act = static_cast<__nv_bfloat16*>(P->act);
  // Folded LayerNorms: statistics of h per 64-column part (sums, then sums of
  // squares) from the GEMMs that write h; the consumers normalise in their epilogue
  // (rstd * (acc - mean * colsum) + b + W . beta; LayerNorm fp32 statistics as in
  // torch.nn.LayerNorm, the variance as E[x^2] - mean^2).
  const int parts = W / 64;
  bool fold = P->row_stats != nullptr && siglip_fold_enabled() && W % 64 == 0 && row_ssq_parts(T, W) == parts &&
              nz(P->wf_proj) && nz(P->bf_proj) && nz(P->cs_proj);
  for (int l = 0; fold && l < P->depth; ++l) {
    const Pi05SiglipLayer& L = P->layers[l];
    fold = nz(L.wf_qkv) && nz(L.bf_qkv) && nz(L.cs_qkv) && nz(L.wf_fc1) && nz(L.bf_fc1) && nz(L.cs_fc1);
  }
  float* st_sum = P->row_stats;
  float* st_ssq = fold ? P->row_stats + (size_t)parts * T : nullptr;
  auto producer = [&](SkinnyParams& sp) {
    if (!fold) return;
    sp.row_ssq = st_ssq;
    sp.row_sum = st_sum;
    sp.ssq_ld = T;
  };
  auto consumer = [&](SkinnyParams& sp, const float* folded_bias, const float* colsum) {
    sp.fold_ssq = st_ssq;
    sp.ln_sum = st_sum;
    sp.fold_parts = parts;
    sp.fold_ld = T;
    sp.fold_d = W;
    sp.fold_eps = P->eps;
    sp.ln_colsum = colsum;
    sp.bias = folded_bias;
  };
  const size_t total = (size_t)T * P->k_pad;
  int rc = launch_pdl(im2col_kernel, dim3((unsigned)std::min<size_t>((total + 255) / 256, 148 * 16)), dim3(256), 0,
                      st, pdl_enabled(), P->images, V, P->image_size, P->patch, P->k_pad,
                      static_cast<__nv_bfloat16*>(P->cols));
  if (rc) return rc;
  {
    SkinnyParams sp = base_params(ws);
    sp.m_tok = T;
    sp.k = P->k_pad;
    sp.n_tiles = W / 128;
    sp.out = h;
    sp.ldo = W;
    sp.bias = P->b_patch;
    sp.pos = P->pos_emb;
    sp.pos_rows = S;
    producer(sp);
    rc = skinny_gemm_run(SK_EPI_STORE, sp, P->w_patch, P->w_patch, W, W, P->cols, P->k_pad, 0, stream);
    if (rc) return rc;
  }
  for (int l = 0; l < P->depth; ++l) {
    const Pi05SiglipLayer& L = P->layers[l];
    if (!fold) rc = pi05_layer_norm(h, L.ln1_w, L.ln1_b, xn, W, T, W, P->eps, stream);
    if (rc) return rc;
    {
      SkinnyParams sp = base_params(ws);
      sp.m_tok = T;
      sp.k = W;
      sp.n_tiles = 3 * W / 128;
      sp.out = qkv;
      sp.ldo = 3 * W;
      sp.bias = L.b_qkv;
      sp.trace_tag = l * 8 + 0;
      if (fold) consumer(sp, L.bf_qkv, L.cs_qkv);
      const void* wq = fold ? L.wf_qkv : L.w_qkv;
      rc = skinny_gemm_run(SK_EPI_STORE, sp, wq, wq, 3 * W, 3 * W, fold ? h : xn, W, 0, stream);
      if (rc) return rc;
    }
    rc = siglip_attention_run(qkv, V, S, W, P->n_heads, P->head_dim, attn, stream, ws.status);
    if (rc) return rc;
    {
      SkinnyParams sp = base_params(ws);
      sp.m_tok = T;
      sp.k = W;
      sp.n_tiles = W / 128;
      sp.out = h;
      sp.ldo = W;
      sp.resid = h;
      sp.ldr = W;
      sp.bias = L.b_o;
      sp.trace_tag = l * 8 + 1;
      producer(sp);
      rc = skinny_gemm_run(SK_EPI_GATED_RESID, sp, L.w_o, L.w_o, W, W, attn, W, 0, stream);
      if (rc) return rc;
    }
    if (!fold) rc = pi05_layer_norm(h, L.ln2_w, L.ln2_b, xn, W, T, W, P->eps, stream);
    if (rc) return rc;
    {
      SkinnyParams sp = base_params(ws);
      sp.m_tok = T;
      sp.k = W;
      sp.n_tiles = (F + 127) / 128;
      sp.n_valid = F;
      sp.out = act;
      sp.ldo = F;
      sp.bias = L.b_fc1;
      sp.act = 1;
      sp.trace_tag = l * 8 + 2;
      if (fold) consumer(sp, L.bf_fc1, L.cs_fc1);
      const void* w1 = fold ? L.wf_fc1 : L.w_fc1;
      rc = skinny_gemm_run(SK_EPI_STORE, sp, w1, w1, F, F, fold ? h : xn, W, 0, stream);
      if (rc) return rc;
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
      sp.bias = L.b_fc2;
      sp.trace_tag = l * 8 + 3;
      producer(sp);
      rc = skinny_gemm_run(SK_EPI_GATED_RESID, sp, L.w_fc2, L.w_fc2, W, W, act, F, 0, stream);
      if (rc) return rc;
    }
  }
  if (!fold) rc = pi05_layer_norm(h, P->post_ln_w, P->post_ln_b, xn, W, T, W, P->eps, stream);
  if (rc) return rc;
  SkinnyParams sp = base_params(ws);
  sp.m_tok = T;
  sp.k = W;
  sp.n_tiles = P->proj_dim / 128;
  sp.out = static_cast<__nv_bfloat16*>(P->out);
  sp.ldo = P->ldo;
  sp.bias = P->b_proj;
  if (fold) consumer(sp, P->bf_proj, P->cs_proj);
  const void* wp = fold ? P->wf_proj : P->w_proj;
  return skinny_gemm_run(SK_EPI_STORE, sp, wp, wp, P->proj_dim, P->proj_dim, fold ? h : xn, W, 0, stream);
}

}  // extern "C"
