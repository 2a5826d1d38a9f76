// Internal interface of the MQA flash attention (see attention.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
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
  int static_rows = 0;                 // keys [0, static_rows) (K, V and mask) do not depend on the
                                       // previous kernel: prefetched before the grid-dependency wait
  int splits = 1;                      // set by the launcher
  int nbuf = 2;                        // set by the launcher: K/V chunk buffers (1 when a split has one chunk)
  int* status = nullptr;               // device status word (bounded-wait timeouts)
  unsigned long long* trace = nullptr; // optional per-CTA timestamps (same format as the GEMMs)
  int trace_tag = 0;
  float* part_o = nullptr;             // [batch][splits, part_rows, head_dim]
  float* part_ml = nullptr;            // [batch][splits, part_rows, 2]
  int part_rows = 0;                   // row pitch of one split's partials (>= rows)
  // Independent observations (mma.sync kernel only): observation z uses q + z * q_batch,
  // k / v + z * kv_batch, key_valid + z * valid_batch and out + z * out_batch
  // (elements), with the same rows / kv_len each.
  int batch = 1;
  size_t q_batch = 0;
  size_t kv_batch = 0;
  size_t valid_batch = 0;
  size_t out_batch = 0;
  int cluster_merge = 0;  // set by the launcher: the tcgen05 kernel's two key splits merge on 2-CTA clusters
};

// splits <= 0 picks a split count that covers the SMs.  head_dim 256 runs on the
// tcgen05 kernel (attention_tc.cu) unless PI05_ATTN_TC=0 selects the mma.sync one.
int mqa_attention_run(AttnParams p, float* part, size_t part_bytes, int splits, void* stream);

// tcgen05 kernel; `combine` launches the split-KV merge when splits > 1.
int mqa_tc_attention_run(AttnParams p, float* part, size_t part_bytes, int splits, cudaStream_t stream,
                         int (*combine)(const AttnParams&, cudaStream_t));
bool tc_attention_enabled();

}  // namespace pi05
