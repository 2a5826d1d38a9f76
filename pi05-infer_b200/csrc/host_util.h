// Host-side helpers shared by the C-ABI translation units: tensor-map encoding
// through the driver entry point (no link against libcuda), PDL launches, error
// text, workspace layout.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <cstring>

#include "pi05_status.h"

namespace pi05 {

// Workspace layout (caller-allocated, 256-byte aligned, zero-filled once):
//   [0, 64)                      device status word (int32 at offset 0) + reserved
//   [64, 64 + 16 KiB)            split-K tile barriers (2 x int32 per tile); zero between launches
//   [kWsAccumOffset, +40 MiB)    fp32 split-K partials (scratch)
//   [kWsStatsOffset, +64 KiB)    fp32 per-row sums of squares for the fused norms (two buffers)
//   [kWsScratchOffset, end)      free scratch (split-KV attention partials, table build)
constexpr size_t kWsStatusOffset = 0;
constexpr size_t kWsCounterOffset = 64;
constexpr int kWsMaxCounters = 4096;
// The top counters are the producer-side norm tickets (one per token slice).
constexpr int kWsNormTicketBase = kWsMaxCounters - 64;
constexpr size_t kWsAccumOffset = 64 + kWsMaxCounters * 4 + 192;  // 16640, 256-aligned
constexpr size_t kWsAccumBytes = size_t(40) << 20;
constexpr size_t kWsStatsOffset = kWsAccumOffset + kWsAccumBytes;
constexpr size_t kWsStatsBytes = size_t(64) << 10;
constexpr size_t kWsScratchOffset = kWsStatsOffset + kWsStatsBytes;

struct Workspace {
  int* status = nullptr;
  int* counters = nullptr;
  float* accum = nullptr;
  size_t accum_bytes = 0;
  float* stats = nullptr;  // kWsStatsBytes
  float* scratch = nullptr;
  size_t scratch_bytes = 0;
};

inline int split_workspace(void* ws, size_t bytes, Workspace* out) {
  if (ws == nullptr || bytes < kWsScratchOffset) return PI05_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return PI05_ERR_ALIGN;
  char* b = static_cast<char*>(ws);
  out->status = reinterpret_cast<int*>(b + kWsStatusOffset);
  out->counters = reinterpret_cast<int*>(b + kWsCounterOffset);
  out->accum = reinterpret_cast<float*>(b + kWsAccumOffset);
  out->accum_bytes = kWsAccumBytes;
  out->stats = reinterpret_cast<float*>(b + kWsStatsOffset);
  out->scratch = reinterpret_cast<float*>(b + kWsScratchOffset);
  out->scratch_bytes = bytes - kWsScratchOffset;
  return PI05_OK;
}

void set_last_error(const char* fmt, ...);
const char* get_last_error();

// Encode a 2-D bf16 row-major tensor map: `rows` x `cols` elements, row pitch
// `ld` elements, box `box_rows` x `box_cols`, 128-byte swizzle (box_cols * 2 == 128).
int make_tmap_bf16_2d(CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                      uint32_t box_rows, uint32_t box_cols, bool swizzle128);

// Same for fp32 elements (box_cols * 4 == 128 with the swizzle).
int make_tmap_f32_2d(CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                     uint32_t box_rows, uint32_t box_cols, bool swizzle128);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Buffer set by pi05_debug_set_trace (per-CTA GEMM timestamps), or nullptr.
unsigned long long* debug_trace_buffer();

// Failure-path test hook set by pi05_debug_set_fault (skip_split < 0 = off).
struct DebugFault {
  int skip_split = -1;
  unsigned long long wait_ns = 0;
};
DebugFault debug_fault();

// Count of kernel launches issued by this library (all threads, all devices).
void count_launch();
long long launch_count();

// Launch with the programmatic-stream-serialization attribute so the kernel's
// prologue (barrier init, TMEM alloc, weight prefetch) overlaps the previous
// kernel's tail; kernels call griddepcontrol.wait before touching activations.
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
               Args&&... args) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  count_launch();
  if (e != cudaSuccess) {
    set_last_error("launch failed: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  return PI05_OK;
}

// launch_pdl with a thread-block cluster of `cluster` CTAs.
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                       dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster.x;
  attr[0].val.clusterDim.y = cluster.y;
  attr[0].val.clusterDim.z = cluster.z;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  count_launch();
  if (e != cudaSuccess) {
    set_last_error("cluster launch failed: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  return PI05_OK;
}

// Global switch for PDL launches (on by default; PI05_PDL=0 in the environment disables).
bool pdl_enabled();

}  // namespace pi05
