// pi05_gate_up_geglu_noalloc: the fused gate/up + GeGLU GEMM for callers that may
// not allocate device memory.
//
// pi05_gate_up_geglu needs a caller-provided workspace for its split-K partials,
// barrier counters and status word.  Some hosts cannot hand one over: a robot
// control loop that forbids any allocation once it is running (a cudaMalloc can
// block and synchronise the device, which breaks a fixed control period), or a
// plugin inside a serving framework that owns every device allocation and gives
// a plugin nothing but its input and output tensors.  This variant keeps its
// scratch in a fixed array compiled into the library instead, so the caller only
// passes inputs and outputs.
//
// Limits: m <= 64 activation rows, n <= 16384 output features, k <= 16384,
// n % 64 == 0, k % 64 == 0.  The scratch is 4 MiB of split-K partials plus a
// 4 KiB header (status word and barrier counters), held by every GPU that loads
// the library until the process exits.  When a shape would need more partial
// space, fewer K splits are used (down to one, which needs none).
//
// Device status: the kernel's bounded waits report a timeout into the status
// word of the built-in header.  Each call clears the barrier counters but leaves
// the status word alone, so a timeout stays visible until the caller reads (and
// clears) it with pi05_gate_up_geglu_noalloc_status.
#include <mutex>

#include "../../include/pi05_b200.h"
#include "host_util.h"
#include "skinny_gemm.h"

using namespace pi05;

namespace {

constexpr int kNoAllocMaxM = 64;
constexpr int kNoAllocMaxN = 16384;
constexpr int kNoAllocMaxK = 16384;
constexpr size_t kNoAllocHeaderBytes = 4096;              // status word + barrier counters
constexpr size_t kNoAllocPartialBytes = size_t(4) << 20;  // split-K partials
constexpr int kNoAllocCounters = (kNoAllocHeaderBytes - 64) / sizeof(int);

// The scratch itself.  Host code must not use this name as a pointer: on the
// host it is only a stand-in for the device symbol.  The device address is
// obtained once per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocHeaderBytes + kNoAllocPartialBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {nullptr};

// Device address of the scratch for the current device (resolved on first use).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error("gate_up_geglu_noalloc: no current device (%s)", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_last_error("gate_up_geglu_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return PI05_ERR_LAUNCH;
    }
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return PI05_OK;
}

}  // namespace

extern "C" int pi05_gate_up_geglu_noalloc(const void* x, const void* wg, const void* wu, void* out, int m, int n,
                                          int k, void* stream) {
  if (x == nullptr || wg == nullptr || wu == nullptr || out == nullptr) {
    set_last_error("gate_up_geglu_noalloc: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (m <= 0 || n <= 0 || k <= 0 || n % 64 || k % 64) {
    set_last_error("gate_up_geglu_noalloc: need n %% 64 == 0, k %% 64 == 0 (m=%d n=%d k=%d)", m, n, k);
    return PI05_ERR_SHAPE;
  }
  if (m > kNoAllocMaxM || n > kNoAllocMaxN || k > kNoAllocMaxK) {
    set_last_error("gate_up_geglu_noalloc: shape m=%d n=%d k=%d exceeds the built-in scratch limits "
                   "(m <= %d, n <= %d, k <= %d); use pi05_gate_up_geglu with a workspace",
                   m, n, k, kNoAllocMaxM, kNoAllocMaxN, kNoAllocMaxK);
    return PI05_ERR_SHAPE;
  }
  if (!aligned16(x) || !aligned16(wg) || !aligned16(wu) || !aligned16(out)) {
    set_last_error("gate_up_geglu_noalloc: pointers must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  void* base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // The barrier counters must start at zero; a call that gave up on a wait could
  // have left them otherwise.  The status word (bytes 0..63) is kept until read;
  // the partials need no clearing.
  cudaError_t e = cudaMemsetAsync(static_cast<char*>(base) + 64, 0, kNoAllocHeaderBytes - 64, st);
  if (e != cudaSuccess) {
    set_last_error("gate_up_geglu_noalloc: clearing the scratch header failed: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  char* b = static_cast<char*>(base);
  SkinnyParams p;
  p.status = reinterpret_cast<int*>(b);
  p.counters = reinterpret_cast<int*>(b + 64);
  p.accum = reinterpret_cast<float*>(b + kNoAllocHeaderBytes);
  p.accum_bytes = kNoAllocPartialBytes;
  p.m_tok = m;
  p.k = k;
  p.n_tiles = n / 64;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = n;
  p.allow_cluster = 0;  // partials go through the built-in scratch
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Same split choice as the workspace entry point, reduced until the partials fit.
  int splits = skinny_choose_splits(p.n_tiles, k / 64, 1, sms);
  const size_t per_split = (size_t)p.n_tiles * 64 * 128 * sizeof(float);
  while (splits > 1 && (size_t)splits * per_split > kNoAllocPartialBytes) --splits;
  if (2 * p.n_tiles > kNoAllocCounters) splits = 1;
  return skinny_gemm_run(SK_EPI_GEGLU, p, wg, wu, n, n, x, k, splits, stream);
}

extern "C" int pi05_gate_up_geglu_noalloc_status(int* host_status, void* stream) {
  if (host_status == nullptr) {
    set_last_error("gate_up_geglu_noalloc_status: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  void* base = nullptr;
  int rc = scratch_address(&base);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, base, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(base, 0, sizeof(int), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_last_error("gate_up_geglu_noalloc_status: status read failed: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  *host_status = v;
  if (v != 0) {
    set_last_error("gate_up_geglu_noalloc: device status word 0x%x (a kernel wait timed out)", v);
    return PI05_ERR_DEVICE;
  }
  return PI05_OK;
}
