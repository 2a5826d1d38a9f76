// Internal interface of the MQA flash attention (see attention.cu).
#pragma once

#include <cuda_bf16.h>
#include <stddef.h>
#include <stdint.h>

namespace pi05 {

struct AttnParams {
  const __nv_bfloat16* q = nullptr;  // [rows, q_stride]: row r = (token, head) pair
  int q_stride = 0;
  const __nv_bfloat16* k = nullptr;  // [kv_len, kv_stride] (one KV head)
  const __nv_bfloat16* v = nullptr;
  int kv_stride = 0;
  const uint8_t* key_valid = nullptr;  // [kv_len], nonzero = attend
  __nv_bfloat16* out = nullptr;        // [rows, out_stride]
  int out_stride = 0;
  int rows = 0;
  int kv_len = 0;
  int head_dim = 0;
  float scale = 0.f;
  int splits = 1;                      // set by the launcher
  float* part_o = nullptr;             // [splits, rows, head_dim]
  float* part_ml = nullptr;            // [splits, rows, 2]
};

// splits <= 0 picks a split count that covers the SMs.
int mqa_attention_run(AttnParams p, float* part, size_t part_bytes, int splits, void* stream);

}  // namespace pi05
