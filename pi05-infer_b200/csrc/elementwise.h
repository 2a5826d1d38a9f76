// Internal interface of the small kernels (see elementwise.cu).
#pragma once

#include <stdint.h>

namespace pi05 {

// mod != null: adaRMS with mod = [scale | shift | gate] (fp32, 3*d); else plain RMSNorm with weight w (fp32, d).
int rms_norm_run(const void* x, int ldx, const float* mod, const float* w, void* out, int ldo, int rows, int d,
                 float eps, void* stream);
// ssq (optional): sum of squares of the bf16 outputs per token and 128-column
// part, ssq[part * ssq_ld + t] (parts = ceil(dout / 128)).  din <= 64.
int action_in_run(const float* x, const float* w, const float* b, void* h, int rows, int din, int dout,
                  void* stream, float* ssq = nullptr, int ssq_ld = 0);
// ssq[part * ld + row] = sum of x^2 over each part_cols-column part of a row (d <= 2048).
int row_ssq_run(const void* x, int ldx, int rows, int d, int part_cols, float* ssq, int ld, void* stream);
// w_out = bf16(w * (1 + scale)) column-wise, b_out = w . shift (fp32); w [rows, k], k % 8 == 0.
int fold_adarms_run(const void* w, int rows, int k, const float* scale, const float* shift, void* w_out,
                    float* b_out, void* stream);
// Final adaRMS + action_out_proj + the sampler update of x_t (d == 1024).  coefs (host, or null =
// flow_ode): {x0 weight, x1 weight, std}; noise [rows, dout] is added times std.
int final_euler_run(const void* h, const float* mod, const float* w, const float* b, float* x_t, float* v_out,
                    int rows, int d, int dout, float eps, float t, float delta, void* stream,
                    const float* coefs = nullptr, const float* noise = nullptr);
int rope_table_run(const uint8_t* valid, int n_prefix, int mode, int rows, const float* inv_freq, int d, void* cos,
                   void* sin, void* stream);
int sinusoid_run(const float* ts, int n_t, int dim, double min_p, double max_p, float* out, void* stream);
// Batched denoise: staging rows (b * tokens + t) of K and V -> row krow0 + t of
// observation b's cache ([batch][kv_rows][d]).
int kv_scatter_run(const void* stage_k, const void* stage_v, void* k_cache, void* v_cache, int batch, int tokens,
                   int krow0, int kv_rows, int d, void* stream);
int linear_f32_rows_run(const float* in, int n_rows, int k, const float* w, const float* b, float* out, int n,
                        int act, void* stream);

}  // namespace pi05
