// extern "C" entry points (declared in include/pi05_b200.h).  Host-side
// validation happens here; kernels live in the other translation units.
#include <algorithm>
#include <atomic>

#include "../../include/pi05_b200.h"
#include "host_util.h"
#include "skinny_gemm.h"

using namespace pi05;

namespace {

std::atomic<int> g_split_override{0};
std::atomic<unsigned long long*> g_trace{nullptr};
std::atomic<int> g_fault_split{-1};
std::atomic<unsigned long long> g_fault_wait_ns{0};

inline bool nz(const void* p) { return p != nullptr; }

int ws_for_skinny(void* ws, size_t bytes, SkinnyParams* p) {
  Workspace w;
  int rc = split_workspace(ws, bytes, &w);
  if (rc) {
    set_last_error("workspace missing, too small or not 256-byte aligned");
    return rc;
  }
  p->status = w.status;
  p->counters = w.counters;
  p->accum = w.accum;
  p->accum_bytes = w.accum_bytes;
  p->trace = g_trace.load();
  return PI05_OK;
}

}  // namespace

namespace pi05 {
unsigned long long* debug_trace_buffer() { return g_trace.load(); }
DebugFault debug_fault() {
  DebugFault f;
  f.skip_split = g_fault_split.load();
  f.wait_ns = g_fault_wait_ns.load();
  return f;
}
}  // namespace pi05

extern "C" {

int pi05_abi_version(void) { return 2; }

const char* pi05_last_error(void) { return get_last_error(); }

size_t pi05_workspace_bytes(int max_tokens, int max_kv) {
  max_tokens = std::max(max_tokens, 1);
  max_kv = std::max(max_kv, 1);
  const int tok = max_tokens <= 64 ? 64 : (max_tokens <= 128 ? 128 : 256);
  const size_t tok_tiles = (max_tokens + tok - 1) / tok;
  (void)tok_tiles;
  // Split-KV attention partials: rows = tokens x 8 heads, up to 32 splits, O + (m, l);
  // the table build needs 3 x 16 x 4096 floats.
  const size_t rows = (size_t)max_tokens * 8;
  const size_t attn = rows * 32 * (256 + 2) * sizeof(float);
  const size_t need = kWsScratchOffset + std::max(attn, (size_t)3 * 16 * 4096 * sizeof(float));
  (void)max_kv;
  return (need + 4095) & ~size_t(4095);
}

int pi05_read_device_status(void* workspace, int* host_status, void* stream) {
  if (!nz(workspace) || !nz(host_status)) return PI05_ERR_INVALID_ARG;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(int), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    set_last_error("status read failed: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  *host_status = v;
  if (v != 0) {
    // A kernel that gave up on a wait may have left split-K counters armed.
    e = cudaMemsetAsync(static_cast<char*>(workspace) + kWsCounterOffset, 0, kWsMaxCounters * sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    set_last_error("device status word 0x%x (kernel wait timed out)%s", v,
                   e == cudaSuccess ? "" : "; resetting the split-K counters failed");
    return PI05_ERR_DEVICE;
  }
  return PI05_OK;
}

long long pi05_launch_count(void) { return launch_count(); }

void pi05_debug_set_splits(int splits) { g_split_override.store(std::max(0, splits)); }

void pi05_debug_set_trace(unsigned long long* buf) { g_trace.store(buf); }

void pi05_debug_set_fault(int skip_split, unsigned long long wait_ns) {
  g_fault_wait_ns.store(wait_ns);
  g_fault_split.store(skip_split < 0 ? -1 : skip_split);
}

int pi05_gate_up_geglu(const void* x, const void* wg, const void* wu, void* out, int m, int n, int k,
                       void* workspace, size_t workspace_bytes, void* stream) {
  if (!nz(x) || !nz(wg) || !nz(wu) || !nz(out)) {
    set_last_error("gate_up_geglu: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (m <= 0 || n <= 0 || k <= 0 || n % 64 || k % 64) {
    set_last_error("gate_up_geglu: need n %% 64 == 0, k %% 64 == 0 (m=%d n=%d k=%d)", m, n, k);
    return PI05_ERR_SHAPE;
  }
  if (!aligned16(x) || !aligned16(wg) || !aligned16(wu) || !aligned16(out)) {
    set_last_error("gate_up_geglu: pointers must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  SkinnyParams p;
  int rc = ws_for_skinny(workspace, workspace_bytes, &p);
  if (rc) return rc;
  p.m_tok = m;
  p.k = k;
  p.n_tiles = n / 64;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = n;
  return skinny_gemm_run(SK_EPI_GEGLU, p, wg, wu, n, n, x, k, g_split_override.load(), stream);
}

int pi05_qkv_rope_kv(const void* x, const void* w, const void* cos, const void* sin, void* q_out, void* k_cache,
                     void* v_cache, int m, int k, int krow0, int kv_rows, int n_q_heads, int n_kv_heads,
                     int head_dim, void* workspace, size_t workspace_bytes, void* stream) {
  if (!nz(x) || !nz(w) || !nz(cos) || !nz(sin) || !nz(q_out) || !nz(k_cache) || !nz(v_cache)) {
    set_last_error("qkv_rope_kv: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (m <= 0 || k <= 0 || k % 64 || head_dim <= 0 || head_dim % 128 || n_q_heads <= 0 || n_kv_heads <= 0 ||
      krow0 < 0 || krow0 + m > kv_rows) {
    set_last_error("qkv_rope_kv: bad shape m=%d k=%d d=%d krow0=%d kv_rows=%d", m, k, head_dim, krow0, kv_rows);
    return PI05_ERR_SHAPE;
  }
  if (!aligned16(x) || !aligned16(w) || !aligned16(cos) || !aligned16(sin) || !aligned16(q_out) ||
      !aligned16(k_cache) || !aligned16(v_cache)) {
    set_last_error("qkv_rope_kv: all tensors must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  SkinnyParams p;
  int rc = ws_for_skinny(workspace, workspace_bytes, &p);
  if (rc) return rc;
  const int rows = (n_q_heads + 2 * n_kv_heads) * head_dim;
  p.m_tok = m;
  p.k = k;
  p.n_tiles = (n_q_heads + n_kv_heads) * (head_dim / 128) + n_kv_heads * head_dim / 128;
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  p.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  p.kv_head_stride = (size_t)kv_rows * head_dim;
  p.krow0 = krow0;
  p.n_q_heads = n_q_heads;
  p.n_kv_heads = n_kv_heads;
  p.head_dim = head_dim;
  return skinny_gemm_run(SK_EPI_QKV_ROPE, p, w, w, rows, rows, x, k, g_split_override.load(), stream);
}

int pi05_linear_gated_residual(const void* x, const void* w, const void* resid, const float* gate, void* out,
                               int m, int n, int k, void* workspace, size_t workspace_bytes, void* stream) {
  if (!nz(x) || !nz(w) || !nz(resid) || !nz(out)) {
    set_last_error("linear_gated_residual: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (m <= 0 || n <= 0 || k <= 0 || n % 128 || k % 64) {
    set_last_error("linear_gated_residual: need n %% 128 == 0, k %% 64 == 0 (n=%d k=%d)", n, k);
    return PI05_ERR_SHAPE;
  }
  if (!aligned16(x) || !aligned16(w) || !aligned16(resid) || !aligned16(out) || (gate && !aligned16(gate))) {
    set_last_error("linear_gated_residual: all tensors must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  SkinnyParams p;
  int rc = ws_for_skinny(workspace, workspace_bytes, &p);
  if (rc) return rc;
  p.m_tok = m;
  p.k = k;
  p.n_tiles = n / 128;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = n;
  p.resid = static_cast<const __nv_bfloat16*>(resid);
  p.ldr = n;
  p.gate = gate;
  return skinny_gemm_run(SK_EPI_GATED_RESID, p, w, w, n, n, x, k, g_split_override.load(), stream);
}

int pi05_linear(const void* x, const void* w, void* out, int m, int n, int k, void* workspace,
                size_t workspace_bytes, void* stream) {
  if (!nz(x) || !nz(w) || !nz(out)) {
    set_last_error("linear: null pointer");
    return PI05_ERR_INVALID_ARG;
  }
  if (m <= 0 || n <= 0 || k <= 0 || n % 128 || k % 64) {
    set_last_error("linear: need n %% 128 == 0, k %% 64 == 0 (n=%d k=%d)", n, k);
    return PI05_ERR_SHAPE;
  }
  if (!aligned16(x) || !aligned16(w) || !aligned16(out)) {
    set_last_error("linear: all tensors must be 16-byte aligned");
    return PI05_ERR_ALIGN;
  }
  SkinnyParams p;
  int rc = ws_for_skinny(workspace, workspace_bytes, &p);
  if (rc) return rc;
  p.m_tok = m;
  p.k = k;
  p.n_tiles = n / 128;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = n;
  return skinny_gemm_run(SK_EPI_STORE, p, w, w, n, n, x, k, g_split_override.load(), stream);
}

}  // extern "C"
