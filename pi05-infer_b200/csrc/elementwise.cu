// Small kernels around the GEMMs: adaRMS / RMS norms, the RoPE table, the action
// in/out projections with the Euler update, and the timestep-conditioning table.
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>

#include "elementwise.h"
#include "host_util.h"
#include "ptx.cuh"

namespace pi05 {
namespace {

// 8 consecutive fp32 / bf16 values (16-byte aligned) into registers.
__device__ __forceinline__ void ew_load8f(const float* src, float* f) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(src));
  const float4 c = __ldg(reinterpret_cast<const float4*>(src + 4));
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = c.x; f[5] = c.y; f[6] = c.z; f[7] = c.w;
}

__device__ __forceinline__ void ew_unpack8(const uint4& u, float* f) {
  const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = __bfloat162float(v[j]);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// adaRMS (modeling_gemma.py:82-116) / Gemma RMSNorm (:94-99):
//   n = x * rsqrt(mean(x^2) + eps)                     fp32
//   ada:   out = bf16(n * (1 + scale) + shift)          mod = [scale | shift | gate] fp32
//   plain: out = bf16(n * (1 + w))
__global__ void __launch_bounds__(256) rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                                       const float* __restrict__ mod, const float* __restrict__ w,
                                                       __nv_bfloat16* __restrict__ out, int ldo, int d, float eps) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int row = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)row * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = __bfloat162float(b[j]);
      ss += f * f;
    }
  }
  const float var = block_sum(ss, red) / (float)d;
  const float rstd = rsqrtf(var + eps);
  for (int i = threadIdx.x * 8; i < d; i += blockDim.x * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + i);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float n = __bfloat162float(b[j]) * rstd;
      float y;
      if (mod != nullptr) y = n * (1.0f + mod[i + j]) + mod[d + i + j];
      else y = n * (1.0f + w[i + j]);
      o[j] = __float2bfloat16(y);
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * ldo + i) = *reinterpret_cast<const uint4*>(o);
  }
}

// action_in_proj (pi0_pytorch.py:303-323): h[t, n] = bf16(sum_k x[t, k] w[n, k] + b[n]), fp32 math.
// ssq (optional): ssq[t] = sum_n bf16(h[t, n])^2, the row statistics of the first
// input_layernorm for the folded-norm q|k|v GEMM.
// action_in_proj on (token, 128-column part) CTAs of 128 threads, one output per
// thread: h[t, n] = bf16(b[n] + sum_k x[t, k] * w[n, k]) with the sum taken in k
// order (fp32).  The part's weight rows are staged in shared memory (row pitch
// din + 1 floats: thread n reads row n with no bank conflict) before the
// grid-dependency wait, since they do not depend on the previous kernel; only the
// token's x row does.  ssq (optional) receives the sum of squares of the part's
// bf16 outputs at ssq[part * ssq_ld + t], the folded input norm's row statistics.
constexpr int kActionInCols = 128;
constexpr int kActionInMaxDin = 64;

__global__ void __launch_bounds__(kActionInCols) action_in_kernel(const float* __restrict__ x,
                                                                  const float* __restrict__ w,
                                                                  const float* __restrict__ b,
                                                                  __nv_bfloat16* __restrict__ h,
                                                                  float* __restrict__ ssq, int ssq_ld, int din,
                                                                  int dout, int vec) {
  __shared__ float ws[kActionInCols * (kActionInMaxDin + 1)];
  __shared__ float xs[kActionInMaxDin];
  __shared__ float red[32];
  const int t = blockIdx.x, n0 = blockIdx.y * kActionInCols;
  const int rows = min(kActionInCols, dout - n0), pitch = din + 1;
  if (vec) {  // din % 4 == 0, w 16-byte aligned
    // All of the thread's float4 loads in flight before the first store.
    constexpr int kPer = kActionInCols * kActionInMaxDin / 4 / kActionInCols;
    const int n4 = rows * din / 4;
    const float4* w4 = reinterpret_cast<const float4*>(w + (size_t)n0 * din);
    float4 v[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = threadIdx.x + j * kActionInCols;
      if (i < n4) v[j] = __ldg(w4 + i);
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int i = threadIdx.x + j * kActionInCols;
      if (i < n4) {
        const int r = (4 * i) / din, k = 4 * i - r * din;
        float* dst = ws + r * pitch + k;
        dst[0] = v[j].x;
        dst[1] = v[j].y;
        dst[2] = v[j].z;
        dst[3] = v[j].w;
      }
    }
  } else {
    for (int i = threadIdx.x; i < rows * din; i += blockDim.x) {
      const int r = i / din, k = i - r * din;
      ws[r * pitch + k] = __ldg(w + (size_t)(n0 + r) * din + k);
    }
  }
  const int n = n0 + threadIdx.x;
  const float bias = threadIdx.x < rows ? __ldg(b + n) : 0.f;
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  for (int k = threadIdx.x; k < din; k += blockDim.x) xs[k] = x[(size_t)t * din + k];
  __syncthreads();
  float ss = 0.f;
  if (threadIdx.x < rows) {
    float acc = bias;
    const float* wr = ws + threadIdx.x * pitch;
    for (int k = 0; k < din; ++k) acc = fmaf(xs[k], wr[k], acc);
    const __nv_bfloat16 o = __float2bfloat16(acc);
    h[(size_t)t * dout + n] = o;
    const float f = __bfloat162float(o);
    ss = f * f;
  }
  if (ssq != nullptr) {
    const float total = block_sum(ss, red);
    if (threadIdx.x == 0) ssq[(size_t)blockIdx.y * ssq_ld + t] = total;
  }
}

// Row statistics of x [rows, d] for a folded RMS norm: ssq[part * ld + row] =
// sum over the part's `part_cols` columns of x^2 (x bf16, fp32 sums).  One CTA per
// row, 8 columns per thread; part_cols is a multiple of 8 and at most 256.
__global__ void __launch_bounds__(256) row_ssq_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int d,
                                                      int part_cols, float* __restrict__ ssq, int ld) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x, c = threadIdx.x * 8;
  float s = 0.f;
  if (c < d) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + (size_t)row * ldx + c);
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = __bfloat162float(b[j]);
      s = fmaf(f, f, s);
    }
  }
  // Sum over the part's threads (part_cols / 8 consecutive lanes, a power of two).
  const int tpp = part_cols / 8;
  for (int o = 1; o < tpp; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (c < d && (threadIdx.x % tpp) == 0) ssq[(size_t)(c / part_cols) * ld + row] = s;
}

// Folds an adaRMS norm (modeling_gemma.py:82-116) into the projection W [rows, k]
// that consumes its output:
//   w_out[n, j] = bf16(W[n, j] * (1 + scale[j])),   b_out[n] = sum_j W[n, j] * shift[j]  (fp32)
// so that W . bf16(h * rstd * (1 + scale) + shift) = rstd * (w_out . h) + b_out up
// to bf16 rounding.  One warp per row, 8 columns per lane and pass.
__global__ void __launch_bounds__(256) fold_adarms_kernel(const __nv_bfloat16* __restrict__ w, int rows, int k,
                                                          const float* __restrict__ scale,
                                                          const float* __restrict__ shift,
                                                          __nv_bfloat16* __restrict__ w_out, float* __restrict__ b_out) {
  const int r = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* wr = w + (size_t)r * k;
  __nv_bfloat16* wo = w_out + (size_t)r * k;
  float acc = 0.f;
  for (int j0 = lane * 8; j0 < k; j0 += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(wr + j0);
    const __nv_bfloat16* bv = reinterpret_cast<const __nv_bfloat16*>(&u);
    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = __bfloat162float(bv[j]);
      o[j] = __float2bfloat16(v * (1.0f + scale[j0 + j]));
      acc = fmaf(v, shift[j0 + j], acc);
    }
    *reinterpret_cast<uint4*>(wo + j0) = *reinterpret_cast<const uint4*>(o);
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) b_out[r] = acc;
}

// Final adaRMS norm -> fp32 -> action_out_proj -> Euler / sampler step
// (modeling_gemma.py:782-783, engine.py:754-767, engine.py:664-675), on (token, 8-output)
// CTAs of d / 8 threads holding 8 columns each (d a multiple of 256, at most 2048):
//   hn[i] = bf16(h[i] * rstd * (1 + scale[i]) + shift[i]),  rstd over the whole row
//   v[j]  = b[j] + sum_i hn[i] * w[j, i]                      (fp32)
//   x_t[j] = (x - v t) wa + (x + v (1 - t)) wb (+ noise[j] sd)
// The weights and the modulation, which do not depend on the previous kernel, are
// read into registers before the grid-dependency wait.
constexpr int kEulerOuts = 8;
constexpr int kEulerMaxThreads = 256;

__global__ void __launch_bounds__(kEulerMaxThreads) final_euler_kernel(const __nv_bfloat16* __restrict__ h,
                                                                    const float* __restrict__ mod,
                                                                    const float* __restrict__ w,
                                                                    const float* __restrict__ b,
                                                                    float* __restrict__ x_t, float* __restrict__ v_out,
                                                                    int d, int dout, float eps, float t, float wa,
                                                                    float wb, float sd,
                                                                    const float* __restrict__ noise) {
  __shared__ float red[32];
  __shared__ float part[kEulerMaxThreads / 32][kEulerOuts];
  const int row = blockIdx.x, j0 = blockIdx.y * kEulerOuts, c = threadIdx.x * 8;
  const int nj = min(kEulerOuts, dout - j0);
  float wr[kEulerOuts][8], sc[8], sh[8];
#pragma unroll
  for (int j = 0; j < kEulerOuts; ++j) {
    if (j < nj) {
      ew_load8f(w + (size_t)(j0 + j) * d + c, wr[j]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) wr[j][i] = 0.f;
    }
  }
  ew_load8f(mod + c, sc);
  ew_load8f(mod + d + c, sh);
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  float hv[8];
  ew_unpack8(*reinterpret_cast<const uint4*>(h + (size_t)row * d + c), hv);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss += hv[i] * hv[i];
  const float rstd = rsqrtf(block_sum(ss, red) / (float)d + eps);
  float acc[kEulerOuts];
#pragma unroll
  for (int j = 0; j < kEulerOuts; ++j) acc[j] = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float hn = bf16_round(hv[i] * rstd * (1.0f + sc[i]) + sh[i]);
#pragma unroll
    for (int j = 0; j < kEulerOuts; ++j) acc[j] = fmaf(hn, wr[j][i], acc[j]);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kEulerOuts; ++j) {
    float v = acc[j];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) part[warp][j] = v;
  }
  __syncthreads();
  if (threadIdx.x < nj) {
    const int j = j0 + threadIdx.x;
    float v = b[j];
    for (int q = 0; q < (int)(blockDim.x >> 5); ++q) v += part[q][threadIdx.x];
    const float x = x_t[(size_t)row * dout + j];
    const float x0 = x - v * t;
    const float x1 = x + v * (1.0f - t);
    float xn = x0 * wa + x1 * wb;
    if (noise != nullptr) xn += noise[(size_t)row * dout + j] * sd;  // stochastic samplers
    x_t[(size_t)row * dout + j] = xn;
    if (v_out != nullptr) v_out[(size_t)row * dout + j] = v;
  }
}

// RoPE table (GemmaRotaryEmbedding, modeling_gemma.py:151-182) for rows whose
// positions derive from the prefix pad mask:
//   mode 0 (prefix): pos[i] = cumsum(valid)[i] - 1         (engine.py:778)
//   mode 1 (suffix): pos[t] = sum(valid[0:n_prefix]) + t     (engine.py:476-477)
__global__ void __launch_bounds__(1024) rope_table_kernel(const uint8_t* __restrict__ valid, int n_prefix, int mode,
                                                          int rows, const float* __restrict__ inv_freq, int d,
                                                          __nv_bfloat16* __restrict__ cos_out,
                                                          __nv_bfloat16* __restrict__ sin_out) {
  __shared__ int cnt[4096];
  __shared__ int wsum[32];
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int n = n_prefix;
  // inclusive scan of valid[0:n] (n <= 4096), 4 elements per thread
  const int per = 4;
  int local[4];
  int run = 0;
  for (int j = 0; j < per; ++j) {
    const int i = threadIdx.x * per + j;
    run += (i < n && valid[i]) ? 1 : 0;
    local[j] = run;
  }
  // warp scan of run totals
  int v = run;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffff, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) wsum[w] = v;
  __syncthreads();
  if (w == 0) {
    int s = wsum[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffff, s, o);
      if (lane >= o) s += u;
    }
    wsum[lane] = s;
  }
  __syncthreads();
  const int excl = v - run + (w > 0 ? wsum[w - 1] : 0);
  for (int j = 0; j < per; ++j) {
    const int i = threadIdx.x * per + j;
    if (i < 4096) cnt[i] = excl + local[j];
  }
  __syncthreads();
  const int total = n > 0 ? cnt[n - 1] : 0;
  const int half = d / 2;
  // Every CTA repeats the (cheap) scan and writes a grid-strided share of the table.
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < rows * d; idx += gridDim.x * blockDim.x) {
    const int r = idx / d, c = idx % d;
    const int pos = (mode == 0) ? cnt[r] - 1 : total + r;
    const float f = (float)pos * inv_freq[c % half];
    cos_out[idx] = __float2bfloat16(cosf(f));
    sin_out[idx] = __float2bfloat16(sinf(f));
  }
}

// torch.linspace(start, end, steps) element, float64 (torch's two-sided formula).
__device__ double linspace_f64(double start, double end, int steps, int i) {
  const double step = (end - start) / (double)(steps - 1);
  return (i < steps / 2) ? start + step * (double)i : end - step * (double)(steps - 1 - i);
}

// create_sinusoidal_pos_embedding (pi0_pytorch.py:29-46): fp64 math, fp32 out.
__global__ void sinusoid_kernel(const float* __restrict__ ts, int n_t, int dim, double min_p, double max_p,
                                float* __restrict__ out) {
  const int half = dim / 2;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n_t * half; idx += gridDim.x * blockDim.x) {
    const int s = idx / half, i = idx % half;
    const double frac = linspace_f64(0.0, 1.0, half, i);
    const double period = min_p * pow(max_p / min_p, frac);
    const double sc = 1.0 / period * 2.0 * 3.141592653589793;
    const double x = sc * (double)ts[s];
    out[(size_t)s * dim + i] = (float)sin(x);
    out[(size_t)s * dim + half + i] = (float)cos(x);
  }
}

// out[s, n] = act(sum_k in[s, k] * w[n, k] + b[n]) for s < n_rows (<= 16), fp32; one warp per n.
// act: 0 = identity, 1 = silu.
__global__ void __launch_bounds__(256) linear_f32_rows_kernel(const float* __restrict__ in, int n_rows, int k,
                                                              const float* __restrict__ w,
                                                              const float* __restrict__ b, float* __restrict__ out,
                                                              int n, int act) {
  extern __shared__ float ins[];  // [n_rows, k]
  for (int i = threadIdx.x; i < n_rows * k; i += blockDim.x) ins[i] = in[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < n; row += warps_total) {
    float acc[16];
#pragma unroll
    for (int s = 0; s < 16; ++s) acc[s] = 0.f;
    const float* wr = w + (size_t)row * k;
    for (int kk = lane; kk < k; kk += 32) {
      const float wv = wr[kk];
#pragma unroll
      for (int s = 0; s < 16; ++s)
        if (s < n_rows) acc[s] = fmaf(ins[s * k + kk], wv, acc[s]);
    }
#pragma unroll
    for (int s = 0; s < 16; ++s) {
      if (s >= n_rows) break;
      float v = acc[s];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
      if (lane == 0) {
        v += (b != nullptr ? b[row] : 0.f);
        if (act == 1) v = v / (1.0f + expf(-v));
        out[(size_t)s * n + row] = v;
      }
    }
  }
}

// Batched denoise: the q|k|v GEMM writes the new K / V rows of all observations to
// a staging buffer [batch * tokens, d] (row b * tokens + t); this copies row
// (b, t) to row krow0 + t of observation b's cache [kv_rows, d].  One thread moves
// 16 bytes.
__global__ void __launch_bounds__(256) kv_scatter_kernel(const __nv_bfloat16* __restrict__ stage_k,
                                                         const __nv_bfloat16* __restrict__ stage_v,
                                                         __nv_bfloat16* __restrict__ k_cache,
                                                         __nv_bfloat16* __restrict__ v_cache, int tokens, int krow0,
                                                         int kv_rows, int d, int total_rows) {
  pdl_wait();
  pdl_launch_dependents();
  const int per_row = d / 8;
  const long n = (long)total_rows * per_row;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int row = (int)(i / per_row), c = (int)(i % per_row) * 8;
    const int b = row / tokens, t = row % tokens;
    const size_t dst = ((size_t)b * kv_rows + krow0 + t) * d + c;
    const size_t src = (size_t)row * d + c;
    *reinterpret_cast<uint4*>(k_cache + dst) = *reinterpret_cast<const uint4*>(stage_k + src);
    *reinterpret_cast<uint4*>(v_cache + dst) = *reinterpret_cast<const uint4*>(stage_v + src);
  }
}

}  // namespace

int rms_norm_run(const void* x, int ldx, const float* mod, const float* w, void* out, int ldo, int rows, int d,
                 float eps, void* stream) {
  if (d % 8 || ldx % 8 || ldo % 8 || rows <= 0) {
    set_last_error("rms_norm: need d, ldx, ldo multiples of 8");
    return PI05_ERR_SHAPE;
  }
  if (!aligned16(x) || !aligned16(out)) {
    set_last_error("rms_norm: x/out must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  return launch_pdl(rms_norm_kernel, dim3(rows), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream),
                    pdl_enabled(), static_cast<const __nv_bfloat16*>(x), ldx, mod, w,
                    static_cast<__nv_bfloat16*>(out), ldo, d, eps);
}

int action_in_run(const float* x, const float* w, const float* b, void* h, int rows, int din, int dout,
                  void* stream, float* ssq, int ssq_ld) {
  if (rows <= 0 || din <= 0 || din > kActionInMaxDin || dout <= 0 || (ssq != nullptr && ssq_ld < rows)) {
    set_last_error("action_in: bad shape rows=%d din=%d (<= %d) dout=%d", rows, din, kActionInMaxDin, dout);
    return PI05_ERR_SHAPE;
  }
  const dim3 grid(rows, (dout + kActionInCols - 1) / kActionInCols);
  return launch_pdl(action_in_kernel, grid, dim3(kActionInCols), 0, reinterpret_cast<cudaStream_t>(stream),
                    pdl_enabled(), x, w, b, static_cast<__nv_bfloat16*>(h), ssq, ssq_ld, din, dout,
                    (din % 4 == 0 && aligned16(w)) ? 1 : 0);
}

int row_ssq_run(const void* x, int ldx, int rows, int d, int part_cols, float* ssq, int ld, void* stream) {
  if (rows <= 0 || d <= 0 || d > 2048 || d % 8 || ldx % 8 || part_cols < 8 || part_cols > 256 ||
      (part_cols & (part_cols - 1)) || d % part_cols || ld < rows || !aligned16(x)) {
    set_last_error("row_ssq: unsupported shape rows=%d d=%d part=%d", rows, d, part_cols);
    return PI05_ERR_SHAPE;
  }
  return launch_pdl(row_ssq_kernel, dim3(rows), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream), pdl_enabled(),
                    static_cast<const __nv_bfloat16*>(x), ldx, d, part_cols, ssq, ld);
}

int fold_adarms_run(const void* w, int rows, int k, const float* scale, const float* shift, void* w_out,
                    float* b_out, void* stream) {
  if (rows <= 0 || k <= 0 || k % 8 != 0) {
    set_last_error("fold_adarms: bad shape rows=%d k=%d (k %% 8 == 0)", rows, k);
    return PI05_ERR_SHAPE;
  }
  if (!aligned16(w) || !aligned16(w_out)) {
    set_last_error("fold_adarms: weights must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  const int blocks = (rows + 7) / 8;
  fold_adarms_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), rows, k, scale, shift, static_cast<__nv_bfloat16*>(w_out), b_out);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("fold_adarms: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  return PI05_OK;
}

int final_euler_run(const void* h, const float* mod, const float* w, const float* b, float* x_t, float* v_out,
                    int rows, int d, int dout, float eps, float t, float delta, void* stream, const float* coefs,
                    const float* noise) {
  if (dout > 64) {
    set_last_error("final_euler: action dim > 64 unsupported");
    return PI05_ERR_SHAPE;
  }
  // flow_ode unless the sampler's weights are given: x0 * (1 - (t - delta)) + x1 * (t - delta)
  const float wa = coefs != nullptr ? coefs[0] : 1.0f - (t - delta);
  const float wb = coefs != nullptr ? coefs[1] : t - delta;
  const float sd = coefs != nullptr ? coefs[2] : 0.0f;
  if (sd != 0.0f && noise == nullptr) {
    set_last_error("final_euler: a stochastic sampler step needs its noise");
    return PI05_ERR_INVALID_ARG;
  }
  if (rows <= 0 || dout <= 0 || d % 256 != 0 || d > 8 * kEulerMaxThreads || !aligned16(h) || !aligned16(w) ||
      !aligned16(mod)) {
    set_last_error("final_euler: width %d must be a multiple of 256 up to %d, h / w / mod 16-byte aligned", d,
                   8 * kEulerMaxThreads);
    return PI05_ERR_SHAPE;
  }
  const dim3 grid(rows, (dout + kEulerOuts - 1) / kEulerOuts);
  return launch_pdl(final_euler_kernel, grid, dim3(d / 8), 0, reinterpret_cast<cudaStream_t>(stream),
                    pdl_enabled(), static_cast<const __nv_bfloat16*>(h), mod, w, b, x_t, v_out, d, dout, eps, t, wa,
                    wb, sd, sd != 0.0f ? noise : nullptr);
}

int rope_table_run(const uint8_t* valid, int n_prefix, int mode, int rows, const float* inv_freq, int d, void* cos,
                   void* sin, void* stream) {
  if (n_prefix > 4096 || (mode == 0 && rows > n_prefix)) {
    set_last_error("rope_table: prefix > 4096 or rows > prefix");
    return PI05_ERR_SHAPE;
  }
  const int blocks = (rows * d + 1023) / 1024;
  const int grid = blocks < 1 ? 1 : (blocks > 148 ? 148 : blocks);
  return launch_pdl(rope_table_kernel, dim3(grid), dim3(1024), 0, reinterpret_cast<cudaStream_t>(stream),
                    pdl_enabled(), valid, n_prefix, mode, rows, inv_freq, d, static_cast<__nv_bfloat16*>(cos),
                    static_cast<__nv_bfloat16*>(sin));
}

int sinusoid_run(const float* ts, int n_t, int dim, double min_p, double max_p, float* out, void* stream) {
  sinusoid_kernel<<<(n_t * dim / 2 + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      ts, n_t, dim, min_p, max_p, out);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("sinusoid: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  return PI05_OK;
}

int linear_f32_rows_run(const float* in, int n_rows, int k, const float* w, const float* b, float* out, int n,
                        int act, void* stream) {
  if (n_rows > 16 || n_rows <= 0 || (size_t)n_rows * k * 4 > 96 * 1024) {
    set_last_error("linear_f32_rows: rows <= 16 and rows*k*4 <= 96 KiB");
    return PI05_ERR_SHAPE;
  }
  const size_t smem = (size_t)n_rows * k * sizeof(float);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(linear_f32_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const int blocks = (n + 7) / 8 < 1184 ? (n + 7) / 8 : 1184;
  linear_f32_rows_kernel<<<blocks, 256, smem, reinterpret_cast<cudaStream_t>(stream)>>>(in, n_rows, k, w, b, out, n,
                                                                                       act);
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error("linear_f32_rows: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  return PI05_OK;
}

int kv_scatter_run(const void* stage_k, const void* stage_v, void* k_cache, void* v_cache, int batch, int tokens,
                   int krow0, int kv_rows, int d, void* stream) {
  if (batch <= 0 || tokens <= 0 || d % 8 != 0 || krow0 < 0 || krow0 + tokens > kv_rows) {
    set_last_error("kv_scatter: bad shape batch=%d tokens=%d krow0=%d kv_rows=%d d=%d", batch, tokens, krow0,
                   kv_rows, d);
    return PI05_ERR_SHAPE;
  }
  const long n = (long)batch * tokens * (d / 8);
  const int grid = (int)std::min<long>((n + 255) / 256, 1184);
  return launch_pdl(kv_scatter_kernel, dim3(grid), dim3(256), 0, reinterpret_cast<cudaStream_t>(stream),
                    pdl_enabled(), static_cast<const __nv_bfloat16*>(stage_k),
                    static_cast<const __nv_bfloat16*>(stage_v), static_cast<__nv_bfloat16*>(k_cache),
                    static_cast<__nv_bfloat16*>(v_cache), tokens, krow0, kv_rows, d, batch * tokens);
}

}  // namespace pi05
