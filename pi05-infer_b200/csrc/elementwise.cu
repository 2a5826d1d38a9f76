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
__global__ void __launch_bounds__(256) action_in_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                        const float* __restrict__ b, __nv_bfloat16* __restrict__ h,
                                                        float* __restrict__ ssq, int din, int dout) {
  extern __shared__ float xs[];
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int t = blockIdx.x;
  for (int k = threadIdx.x; k < din; k += blockDim.x) xs[k] = x[(size_t)t * din + k];
  __syncthreads();
  float ss = 0.f;
  for (int n = threadIdx.x; n < dout; n += blockDim.x) {
    float acc = b[n];
    const float* wr = w + (size_t)n * din;
    for (int k = 0; k < din; ++k) acc = fmaf(xs[k], wr[k], acc);
    const __nv_bfloat16 o = __float2bfloat16(acc);
    h[(size_t)t * dout + n] = o;
    const float f = __bfloat162float(o);
    ss = fmaf(f, f, ss);
  }
  if (ssq != nullptr) {
    const float total = block_sum(ss, red);
    if (threadIdx.x == 0) ssq[t] = total;
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

// Final adaRMS norm -> fp32 -> action_out_proj -> flow_ode Euler step
// (modeling_gemma.py:782-783, engine.py:754-767, engine.py:664-675).
__global__ void __launch_bounds__(256) final_euler_kernel(const __nv_bfloat16* __restrict__ h,
                                                          const float* __restrict__ mod,
                                                          const float* __restrict__ w,
                                                          const float* __restrict__ b, float* __restrict__ x_t,
                                                          float* __restrict__ v_out, int d, int dout, float eps,
                                                          float t, float wa, float wb, float sd,
                                                          const float* __restrict__ noise) {
  extern __shared__ float hn[];  // [d]
  __shared__ float red[32];
  __shared__ float vs[64];
  pdl_wait();
  pdl_launch_dependents();  // let the next kernel's CTAs start their prologue / weight prefetch
  const int row = blockIdx.x;
  const __nv_bfloat16* hr = h + (size_t)row * d;
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float f = __bfloat162float(hr[i]);
    ss += f * f;
  }
  const float rstd = rsqrtf(block_sum(ss, red) / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float n = __bfloat162float(hr[i]) * rstd;
    hn[i] = bf16_round(n * (1.0f + mod[i]) + mod[d + i]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int j = warp; j < dout; j += nw) {
    const float* wr = w + (size_t)j * d;
    float acc = 0.f;
    for (int i = lane; i < d; i += 32) acc = fmaf(hn[i], wr[i], acc);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
    if (lane == 0) vs[j] = acc + b[j];
  }
  __syncthreads();
  if (threadIdx.x < dout) {
    const int j = threadIdx.x;
    const float v = vs[j];
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
                  void* stream, float* ssq) {
  return launch_pdl(action_in_kernel, dim3(rows), dim3(256), din * sizeof(float),
                    reinterpret_cast<cudaStream_t>(stream), pdl_enabled(), x, w, b, static_cast<__nv_bfloat16*>(h),
                    ssq, din, dout);
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
  return launch_pdl(final_euler_kernel, dim3(rows), dim3(256), d * sizeof(float),
                    reinterpret_cast<cudaStream_t>(stream), pdl_enabled(), static_cast<const __nv_bfloat16*>(h), mod,
                    w, b, x_t, v_out, d, dout, eps, t, wa, wb, sd, sd != 0.0f ? noise : nullptr);
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
