// Observation preprocessing and action output transform on the GPU: the work the
// reference does on the host around sample_actions in predict_action_batch
// (engine.py:321-342):
//
//   * camera images, uint8 [N, H, W, 3] (or [N, 3, H, W]) as the environment hands
//     them over, to the model's fp32 [N, 3, S, S] in [-1, 1], resized with padding
//     to S x S when they are not that size already (openpi's image preprocessing;
//     bilinear with half-pixel centres, the aspect ratio kept, the border filled
//     with black = -1);
//   * the robot state normalised with the checkpoint's statistics and zero-padded
//     to the model's action dimension (openpi Normalize + PadStatesAndActions);
//   * the model's actions un-normalised and cut to the robot's action dimension
//     (openpi Unnormalize + the policy's output slice, e.g. LiberoOutputs [:, :7],
//     TurtleOutputs in dataconfig/policies/turtle_policy.py:89-93).
//
// Normalisation (per feature j, stats a/b):
//   mode 0 (mean/std):   y = (x - mean) / (std + 1e-6),      x = y * (std + 1e-6) + mean
//   mode 1 (quantiles):  y = (x - q01) / (q99 - q01 + 1e-6) * 2 - 1,
//                        x = (y + 1) / 2 * (q99 - q01 + 1e-6) + q01
// Features past the statistics' length pass through unchanged.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/pi05_b200.h"
#include "host_util.h"

namespace pi05 {
namespace {

constexpr float kNormEps = 1e-6f;

// One thread per output element (image, channel, y, x).
__global__ void __launch_bounds__(256) preprocess_images_kernel(const uint8_t* __restrict__ src, int n, int h, int w,
                                                                int chw, float* __restrict__ dst, int s, int rh,
                                                                int rw, int pad_y, int pad_x) {
  const long total = (long)n * 3 * s * s;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int x = (int)(i % s);
    const int y = (int)((i / s) % s);
    const int c = (int)((i / ((long)s * s)) % 3);
    const int img = (int)(i / ((long)3 * s * s));
    const int yy = y - pad_y, xx = x - pad_x;
    float v = -1.0f;  // padding: black
    if (yy >= 0 && yy < rh && xx >= 0 && xx < rw) {
      // Source coordinate of the resized pixel centre (half-pixel centres, clamped at 0).
      const float sy = fmaxf(((float)yy + 0.5f) * ((float)h / (float)rh) - 0.5f, 0.0f);
      const float sx = fmaxf(((float)xx + 0.5f) * ((float)w / (float)rw) - 0.5f, 0.0f);
      const int y0 = min((int)sy, h - 1), x0 = min((int)sx, w - 1);
      const int y1 = min(y0 + 1, h - 1), x1 = min(x0 + 1, w - 1);
      const float ly = sy - (float)y0, lx = sx - (float)x0;
      auto px = [&](int yi, int xi) -> float {
        const size_t off = chw ? (((size_t)img * 3 + c) * h + yi) * w + xi : (((size_t)img * h + yi) * w + xi) * 3 + c;
        return (float)src[off];
      };
      const float top = px(y0, x0) * (1.0f - lx) + px(y0, x1) * lx;
      const float bot = px(y1, x0) * (1.0f - lx) + px(y1, x1) * lx;
      const float p = top * (1.0f - ly) + bot * ly;
      v = p / 255.0f * 2.0f - 1.0f;
    }
    dst[i] = v;
  }
}

// Normalise rows of `x` [rows, din] into `out` [rows, dout] (zero past din).
__global__ void normalize_rows_kernel(const float* __restrict__ x, int rows, int din, const float* __restrict__ a,
                                      const float* __restrict__ b, int nstat, int mode, float* __restrict__ out,
                                      int dout) {
  const long total = (long)rows * dout;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int j = (int)(i % dout);
    const long r = i / dout;
    float v = 0.0f;
    if (j < din) {
      v = x[r * din + j];
      if (j < nstat) {
        if (mode == 0)
          v = (v - a[j]) / (b[j] + kNormEps);
        else
          v = (v - a[j]) / (b[j] - a[j] + kNormEps) * 2.0f - 1.0f;
      }
    }
    out[i] = v;
  }
}

// Un-normalise the first dout features of rows of `x` [rows, din] into `out` [rows, dout].
__global__ void unnormalize_rows_kernel(const float* __restrict__ x, int rows, int din, const float* __restrict__ a,
                                        const float* __restrict__ b, int nstat, int mode, float* __restrict__ out,
                                        int dout) {
  const long total = (long)rows * dout;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int j = (int)(i % dout);
    const long r = i / dout;
    float v = x[r * din + j];
    if (j < nstat) {
      if (mode == 0)
        v = v * (b[j] + kNormEps) + a[j];
      else
        v = (v + 1.0f) * 0.5f * (b[j] - a[j] + kNormEps) + a[j];
    }
    out[i] = v;
  }
}

int grid_for(long total) {
  long g = (total + 255) / 256;
  return (int)(g < 1 ? 1 : (g > 4096 ? 4096 : g));
}

}  // namespace
}  // namespace pi05

using namespace pi05;

extern "C" {

int pi05_preprocess_images(const uint8_t* images, int n, int h, int w, int layout, float* out, int size,
                           void* stream) {
  if (images == nullptr || out == nullptr) {
    set_last_error("preprocess_images: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (n <= 0 || h <= 0 || w <= 0 || size <= 0 || size > 4096 || h > 16384 || w > 16384 || (layout != 0 && layout != 1)) {
    set_last_error("preprocess_images: bad shape n=%d h=%d w=%d size=%d layout=%d", n, h, w, size, layout);
    return PI05_ERR_SHAPE;
  }
  // Resize with padding: keep the aspect ratio, fit the longer side.
  const double ratio = (double)w / size > (double)h / size ? (double)w / size : (double)h / size;
  int rh = (int)((double)h / ratio), rw = (int)((double)w / ratio);
  rh = rh < 1 ? 1 : (rh > size ? size : rh);
  rw = rw < 1 ? 1 : (rw > size ? size : rw);
  const int pad_y = (size - rh) / 2, pad_x = (size - rw) / 2;
  const long total = (long)n * 3 * size * size;
  return launch_pdl(preprocess_images_kernel, dim3(grid_for(total)), dim3(256), 0,
                    reinterpret_cast<cudaStream_t>(stream), false, images, n, h, w, layout, out, size, rh, rw, pad_y,
                    pad_x);
}

int pi05_normalize_rows(const float* x, int rows, int din, const float* a, const float* b, int nstat, int mode,
                        float* out, int dout, void* stream) {
  if (x == nullptr || out == nullptr || (nstat > 0 && (a == nullptr || b == nullptr))) {
    set_last_error("normalize_rows: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (rows <= 0 || din <= 0 || dout < din || nstat < 0 || nstat > din || (mode != 0 && mode != 1)) {
    set_last_error("normalize_rows: bad shape rows=%d din=%d dout=%d nstat=%d mode=%d", rows, din, dout, nstat, mode);
    return PI05_ERR_SHAPE;
  }
  return launch_pdl(normalize_rows_kernel, dim3(grid_for((long)rows * dout)), dim3(256), 0,
                    reinterpret_cast<cudaStream_t>(stream), false, x, rows, din, a, b, nstat, mode, out, dout);
}

int pi05_unnormalize_rows(const float* x, int rows, int din, const float* a, const float* b, int nstat, int mode,
                          float* out, int dout, void* stream) {
  if (x == nullptr || out == nullptr || (nstat > 0 && (a == nullptr || b == nullptr))) {
    set_last_error("unnormalize_rows: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (rows <= 0 || din <= 0 || dout <= 0 || dout > din || nstat < 0 || nstat > din || (mode != 0 && mode != 1)) {
    set_last_error("unnormalize_rows: bad shape rows=%d din=%d dout=%d nstat=%d mode=%d", rows, din, dout, nstat,
                   mode);
    return PI05_ERR_SHAPE;
  }
  return launch_pdl(unnormalize_rows_kernel, dim3(grid_for((long)rows * dout)), dim3(256), 0,
                    reinterpret_cast<cudaStream_t>(stream), false, x, rows, din, a, b, nstat, mode, out, dout);
}

}  // extern "C"
