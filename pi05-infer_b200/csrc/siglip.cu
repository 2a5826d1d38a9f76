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
// Attention here is per-head (16 heads x 72 dims, 256 tokens per view, no mask):
// mma.sync flash kernel, head dim zero-padded to 80.
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

// ---- per-head flash attention, head dim 72 (padded to 80), mma.sync --------
constexpr int kHd = 72;
constexpr int kHdPad = 80;
constexpr int kRowE = 88;              // smem row pitch in elements (176 B: conflict-free ldmatrix)
constexpr int kRowB = kRowE * 2;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& a, uint32_t& b) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& a, uint32_t& b) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Grid (views * heads, seq / 64); 4 warps x 16 query rows; all `seq` keys in smem.
// qkv [views*seq, 3*width] (q | k | v, head h at columns h*72), out [views*seq, width].
template <int SEQ>
__global__ void __launch_bounds__(128) mha72_kernel(const __nv_bfloat16* __restrict__ qkv, int width, int heads,
                                                    float scale, __nv_bfloat16* __restrict__ out) {
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);  // 64 x 88
  __nv_bfloat16* sK = sQ + 64 * kRowE;                          // SEQ x 88
  __nv_bfloat16* sV = sK + SEQ * kRowE;                         // SEQ x 88
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int vh = blockIdx.x, view = vh / heads, h = vh % heads;
  const int q0 = blockIdx.y * 64;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t ld = (size_t)3 * width;
  const __nv_bfloat16* base = qkv + (size_t)view * SEQ * ld + h * kHd;
  // 9 chunks of 16 B per 72-element row, copied asynchronously; chunk 9 (columns
  // 72..79) is zero-filled.  Four commit groups: Q with keys 0..63, then keys
  // 64c..64c+63 (K and V rows), so the key loop starts on the first 64 keys while
  // the others are still arriving.
  auto copy_rows = [&](__nv_bfloat16* dst0, const __nv_bfloat16* src0, int rows) {
    for (int i = tid; i < rows * 10; i += 128) {
      const int row = i / 10, c = i % 10;
      const int n = c < 9 ? 16 : 0;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst0 + row * kRowE + c * 8)),
                   "l"(src0 + (size_t)row * ld + (c < 9 ? c * 8 : 0)), "r"(n)
                   : "memory");
    }
  };
  copy_rows(sQ, base + (size_t)q0 * ld, 64);
#pragma unroll
  for (int c = 0; c < SEQ / 64; ++c) {
    copy_rows(sK + c * 64 * kRowE, base + (size_t)(c * 64) * ld + width, 64);
    copy_rows(sV + c * 64 * kRowE, base + (size_t)(c * 64) * ld + 2 * width, 64);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  static_assert(SEQ == 256, "four key groups");
  asm volatile("cp.async.wait_group 3;" ::: "memory");
  __syncthreads();
  const uint32_t aQ = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));
  const uint32_t aK = static_cast<uint32_t>(__cvta_generic_to_shared(sK));
  const uint32_t aV = static_cast<uint32_t>(__cvta_generic_to_shared(sV));
  const int g = lane >> 2, t4 = lane & 3;
  // Q fragments for this warp's 16 rows, 5 k-steps of 16 dims.
  uint32_t qa[5][4];
#pragma unroll
  for (int kk = 0; kk < 5; ++kk) {
    const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int c = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(aQ + (r * kRowE + c) * 2, qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
  }
  float o[10][4];
#pragma unroll
  for (int j = 0; j < 10; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  for (int kc = 0; kc < SEQ; kc += 64) {
    if (kc > 0) {  // keys kc .. kc+63 (groups still in flight after this one: 3 - kc / 64)
      if (kc == 64)
        asm volatile("cp.async.wait_group 2;" ::: "memory");
      else if (kc == 128)
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      else
        asm volatile("cp.async.wait_group 0;" ::: "memory");
      __syncthreads();
    }
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 5; ++kk) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t b0, b1;
        const int r = kc + j * 8 + (lane & 7);
        const int c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x2(aK + (r * kRowE + c) * 2, b0, b1);
        mma_bf16(s[j], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; e += 2) {  // bf16(bf16(q.k) * scale), two values per conversion
        bf16_round2(s[j][e], s[j][e + 1]);
        s[j][e] *= scale;
        s[j][e + 1] *= scale;
        bf16_round2(s[j][e], s[j][e + 1]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) mx[e >> 1] = fmaxf(mx[e >> 1], s[j][e]);
    }
    float corr[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffff, mx[hh], 1));
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffff, mx[hh], 2));
      const float mn = fmaxf(m_run[hh], mx[hh]);
      corr[hh] = __expf(m_run[hh] - mn);
      m_run[hh] = mn;
    }
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = __expf(s[j][e] - m_run[e >> 1]);
        s[j][e] = pv;
        ls[e >> 1] += pv;
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      ls[hh] += __shfl_xor_sync(0xffffffff, ls[hh], 1);
      ls[hh] += __shfl_xor_sync(0xffffffff, ls[hh], 2);
      l_run[hh] = l_run[hh] * corr[hh] + ls[hh];
    }
#pragma unroll
    for (int j = 0; j < 10; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int j = 0; j < 10; ++j) {
        uint32_t b0, b1;
        const int r = kc + kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        ldsm_x2_t(aV + (r * kRowE + j * 8) * 2, b0, b1);
        mma_bf16(o[j], a0, a1, a2, a3, b0, b1);
      }
    }
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float inv = 1.f / l_run[hh];
    const int row = q0 + warp * 16 + g + hh * 8;
    __nv_bfloat16* dst = out + ((size_t)view * SEQ + row) * width + h * kHd;
#pragma unroll
    for (int j = 0; j < 9; ++j)
      *reinterpret_cast<uint32_t*>(dst + j * 8 + 2 * t4) = pack2(o[j][2 * hh] * inv, o[j][2 * hh + 1] * inv);
  }
}

inline bool nz(const void* p) { return p != nullptr; }

int siglip_attention_run(const void* qkv, int views, int seq, int width, int heads, int head_dim, void* out,
                         void* stream) {
  if (!nz(qkv) || !nz(out)) {
    set_last_error("siglip_attention: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (head_dim != kHd || seq != 256 || heads * head_dim != width || views <= 0 || !aligned16(qkv) ||
      !aligned16(out)) {
    set_last_error("siglip_attention: supports head_dim 72, 256 tokens per view, 16-byte aligned buffers");
    return PI05_ERR_SHAPE;
  }
  const size_t smem = (size_t)(64 + 2 * 256) * kRowB;
  static bool attr_done[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_done[dev]) {
    cudaFuncSetAttribute(mha72_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_done[dev] = true;
  }
  return launch_pdl(mha72_kernel<256>, dim3(views * heads, seq / 64), dim3(128), smem,
                    reinterpret_cast<cudaStream_t>(stream), pdl_enabled(), static_cast<const __nv_bfloat16*>(qkv),
                    width, heads, 1.0f / std::sqrt((float)head_dim), static_cast<__nv_bfloat16*>(out));
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
    rc = siglip_attention_run(qkv, V, S, W, P->n_heads, P->head_dim, attn, stream);
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
