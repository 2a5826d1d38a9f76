// Persistent denoise kernel: all Euler steps of the action expert in ONE launch.
//
// At bs=1 the denoise loop is a chain of ~145 dependent phases per step (per
// layer: adaRMS, q|k|v GEMM, attention, combine, o_proj, adaRMS, gate/up, down),
// each far too small to fill the GPU by itself.  Launched as separate kernels,
// every phase pays launch latency, a cold DRAM round trip for its weights and a
// grid-wide drain.  Here one CTA per SM stays resident for the whole loop:
//
//   warp 0      weight TMA: walks this CTA's GEMM units for every layer of every
//               step and streams their weight tiles into a shared-memory ring.
//               Weights never depend on activations, so this warp is only ever
//               held back by free ring slots -- HBM keeps streaming across phase
//               boundaries while the other warps wait on their inputs.
//   warp 1      tcgen05.mma issue into two TMEM accumulators (double buffered).
//   warp 2      activation TMA: waits until a unit's input phase is complete, then
//               loads the activation k-blocks next to the weights in the ring.
//   warps 3-6   workers: GEMM epilogues (split-K publish, tile barrier, fixed-order
//               reduction of a slice, fused RoPE / GeGLU / gated residual), the
//               attention units (mma.sync flash, split-KV), the split combine, the
//               adaRMS rows (with action_in_proj for layer 0) and the final
//               norm + action_out_proj + Euler rows.
//
// Phases are ordered by monotonic completion counters in global memory (acquire
// loads, release increments); no grid-wide barrier.  Every wait is bounded: after
// kWaitTimeoutNs the CTA records a status bit, raises its abort flag and unwinds.
//
// The math of each phase is the same device code as the multi-kernel path
// (gemm_epilogue.cuh, the attention/norm formulas of attention.cu and
// elementwise.cu), so both paths follow the reference's rounding points.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>

#include "../../include/pi05_b200.h"
#include "gemm_epilogue.cuh"
#include "host_util.h"
#include "ptx.cuh"

namespace pi05 {
namespace mega {

using namespace gemm;

constexpr int kMaxLayers = 18;
constexpr int kStages = 5;
constexpr int kTok = 64;                      // UMMA N: tokens (50 valid)
constexpr int kWBytes = kBM * 128;            // 128 weight rows x 64 k
constexpr int kXBytes = kTok * 128;           // 64 tokens x 64 k
constexpr int kStageBytes = kWBytes + kXBytes;
constexpr int kThreads = 224;
constexpr int kWorkerWarp0 = 3;
constexpr int kD = 256;                       // head dim
constexpr int kChunk = 64;                    // keys per attention unit
constexpr int kRowBytes = kD * 2;
constexpr int kAttnSmem = 3 * 64 * kRowBytes; // Q, K, V tiles

enum Phase { PH_NORM1 = 0, PH_QKV, PH_ATTN, PH_COMB, PH_OPROJ, PH_NORM2, PH_GEGLU, PH_DOWN, PH_FINAL, PH_COUNT };
constexpr int kCtrStride = 32;   // ints: each counter on its own 128-byte line
constexpr int kTraceEvents = 20; // stamps per (CTA, iteration)
constexpr int kTraceSlots = 16 * 18 * kTraceEvents + 64;
enum Op { OP_QKV = 0, OP_O = 1, OP_GU = 2, OP_DOWN = 3 };

struct alignas(64) Maps {
  CUtensorMap w[kMaxLayers][5];  // q|k|v, o, gate, up, down
  CUtensorMap x[4];              // xn1 [T, W], attn [T, HQ*D], xn2 [T, W], act [T, F]
};

struct GemmShape {
  int tiles, splits, kb;
};

struct Args {
  int depth, width, mlp, hq, hd, tokens, action_dim, prefix_len, kv_rows, num_steps, n_norm;
  float eps, attn_scale;
  GemmShape g[4];
  int attn_splits, attn_units, comb_units;
  __nv_bfloat16* h;
  __nv_bfloat16* xn1;
  __nv_bfloat16* xn2;
  __nv_bfloat16* q;
  __nv_bfloat16* attn;
  __nv_bfloat16* act;
  const __nv_bfloat16* rope_cos;
  const __nv_bfloat16* rope_sin;
  __nv_bfloat16* k_cache[kMaxLayers];
  __nv_bfloat16* v_cache[kMaxLayers];
  const uint8_t* key_valid;
  const float* mod_table;
  const float* w_in;
  const float* b_in;
  const float* w_out;
  const float* b_out;
  float* x_t;
  float* v_t;
  float ts[17];
  int* done;      // [PH_COUNT] completion counters, one per 128-byte line (zero at launch)
  int* tile_cnt;  // [4][64] split-K tile barriers, one per 128-byte line (zero at launch)
  unsigned long long* trace;  // optional [gridDim][kTraceSlots] globaltimer stamps (null = off)
  float* part[4]; // split-K partials per op: [tiles][splits][kTok][128]
  float* attn_o;  // [attn_splits][rows][256]
  float* attn_ml; // [attn_splits][rows][2]
  int* status;
};

__device__ __forceinline__ bool abort_set(volatile int* f) { return *f != 0; }

// Spin (one thread) until *ctr >= target; false on abort or timeout.
__device__ __forceinline__ bool wait_geq(const int* ctr, int target, volatile int* s_abort, int* status) {
  if (ld_acquire(ctr) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (abort_set(s_abort)) return false;
    __nanosleep(40);
    if (ld_acquire(ctr) >= target) return true;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      report_status(status, PI05_DEV_TIMEOUT_FLAG);
      *s_abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity, volatile int* s_abort, int* status,
                                                int code) {
  if (mbar_try_wait(smem_u32(bar), parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(smem_u32(bar), parity)) return true;
    if (abort_set(s_abort)) return false;
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      report_status(status, code);
      *s_abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void stamp(const Args& a, int it, int ev) {
  if (a.trace != nullptr) a.trace[(size_t)blockIdx.x * kTraceSlots + it * kTraceEvents + ev] = globaltimer_ns();
}

__device__ __forceinline__ void signal(int* ctr) {
  __threadfence();
  atomicAdd(ctr, 1);
}

// SkinnyParams view of one GEMM op of layer l / step modulation `mods`, for the
// shared tile-row mapping and epilogue code.
__device__ __forceinline__ SkinnyParams op_params(const Args& a, int op, int l, const float* mods) {
  SkinnyParams p;
  p.m_tok = a.tokens;
  p.head_dim = a.hd;
  p.n_q_heads = a.hq;
  p.n_kv_heads = 1;
  if (op == OP_QKV) {
    p.cos = a.rope_cos;
    p.sin = a.rope_sin;
    p.q_out = a.q;
    p.k_cache = a.k_cache[l];
    p.v_cache = a.v_cache[l];
    p.kv_head_stride = (size_t)a.kv_rows * a.hd;
    p.krow0 = a.prefix_len;
  } else if (op == OP_O) {
    p.out = a.h;
    p.ldo = a.width;
    p.resid = a.h;
    p.ldr = a.width;
    p.gate = mods + (size_t)(2 * l) * 3 * a.width + 2 * a.width;
  } else if (op == OP_GU) {
    p.out = a.act;
    p.ldo = a.mlp;
  } else {
    p.out = a.h;
    p.ldo = a.width;
    p.resid = a.h;
    p.ldr = a.width;
    p.gate = mods + (size_t)(2 * l + 1) * 3 * a.width + 2 * a.width;
  }
  return p;
}

__device__ __forceinline__ TileRows op_rows(const SkinnyParams& p, int op, int tile) {
  if (op == OP_QKV) return tile_rows<SK_EPI_QKV_ROPE>(p, tile);
  if (op == OP_GU) return tile_rows<SK_EPI_GEGLU>(p, tile);
  return tile_rows<SK_EPI_GATED_RESID>(p, tile);
}

__device__ __forceinline__ const CUtensorMap* wmap(const Maps& m, int l, int op, int box) {
  if (op == OP_QKV) return &m.w[l][0];
  if (op == OP_O) return &m.w[l][1];
  if (op == OP_GU) return &m.w[l][box == 0 ? 2 : 3];
  return &m.w[l][4];
}

// ---------------------------------------------------------------------------
// worker routines (warps 3-6, 128 threads; `et` = 0..127, `wrel` = 0..3)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float worker_sum(float v, float* s_red, int wrel, int lane) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  named_bar_sync(2, 128);
  if (lane == 0) s_red[wrel] = v;
  named_bar_sync(2, 128);
  return s_red[0] + s_red[1] + s_red[2] + s_red[3];
}

// adaRMS of row t (width 1024 = 128 threads x 8); layer 0 first forms the row
// from action_in_proj (fp32 math, bf16 out) and stores it into h.
__device__ void norm_row(const Args& a, int t, bool action_in, const float* mod, __nv_bfloat16* out, float* s_red,
                         int et, int wrel, int lane) {
  const int c0 = et * 8;
  float x[8];
  if (action_in) {
    const float* xt = a.x_t + (size_t)t * a.action_dim;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float* wr = a.w_in + (size_t)(c0 + j) * a.action_dim;
      float acc = a.b_in[c0 + j];
      for (int k = 0; k < a.action_dim; ++k) acc = fmaf(xt[k], wr[k], acc);
      x[j] = bf16_round(acc);
    }
    *reinterpret_cast<uint4*>(a.h + (size_t)t * a.width + c0) = pack8(x);
  } else {
    unpack8(*reinterpret_cast<const uint4*>(a.h + (size_t)t * a.width + c0), x);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
  const float var = worker_sum(ss, s_red, wrel, lane) / (float)a.width;
  const float rstd = rsqrtf(var + a.eps);
  float o[8], sc[8], sh[8];
  load8f(mod + c0, sc);
  load8f(mod + a.width + c0, sh);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = (x[j] * rstd) * (1.0f + sc[j]) + sh[j];
  *reinterpret_cast<uint4*>(out + (size_t)t * a.width + c0) = pack8(o);
}

// Final adaRMS (mod row 2*depth) -> fp32 -> action_out_proj -> Euler update of row t.
__device__ void final_row(const Args& a, int t, const float* mod, float tt, float dt, float* s_hn, float* s_red,
                          int et, int wrel, int lane) {
  const int c0 = et * 8;
  float x[8];
  unpack8(*reinterpret_cast<const uint4*>(a.h + (size_t)t * a.width + c0), x);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
  const float rstd = rsqrtf(worker_sum(ss, s_red, wrel, lane) / (float)a.width + a.eps);
  float sc[8], sh[8];
  load8f(mod + c0, sc);
  load8f(mod + a.width + c0, sh);
#pragma unroll
  for (int j = 0; j < 8; ++j) s_hn[c0 + j] = bf16_round((x[j] * rstd) * (1.0f + sc[j]) + sh[j]);
  named_bar_sync(2, 128);
  float* vs = s_red + 8;  // [action_dim <= 32]
  for (int j = wrel; j < a.action_dim; j += 4) {
    const float* wr = a.w_out + (size_t)j * a.width;
    float acc = 0.f;
    for (int n = lane; n < a.width; n += 32) acc = fmaf(s_hn[n], wr[n], acc);
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
    if (lane == 0) vs[j] = acc + a.b_out[j];
  }
  named_bar_sync(2, 128);
  if (et < a.action_dim) {
    const float v = vs[et];
    float* xp = a.x_t + (size_t)t * a.action_dim + et;
    const float xv = *xp;
    const float x0 = xv - v * tt;
    const float x1 = xv + v * (1.0f - tt);
    *xp = x0 * (1.0f - (tt - dt)) + x1 * (tt - dt);
    if (a.v_t != nullptr) a.v_t[(size_t)t * a.action_dim + et] = v;
  }
  named_bar_sync(2, 128);
}

// ---- attention unit: 64 query rows x one 64-key chunk, partial (O, m, l) -----
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * kRowBytes + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ void attn_unit(const Args& a, int l, int au, uint8_t* sQ, uint8_t* sK, uint8_t* sV, uint8_t* s_valid,
                          int et, int wrel, int lane) {
  const int rows = a.tokens * a.hq;
  const int kv_len = a.prefix_len + a.tokens;
  const int rb = au / a.attn_splits, sp = au % a.attn_splits;
  const int row0 = rb * 64, key0 = sp * kChunk;
  const __nv_bfloat16* kc = a.k_cache[l];
  const __nv_bfloat16* vc = a.v_cache[l];
  const uint32_t qa = smem_u32(sQ), ka = smem_u32(sK), va = smem_u32(sV);
  for (int i = et; i < 64 * 32; i += 128) {
    const int r = i >> 5, c = i & 31;
    const bool okq = row0 + r < rows;
    cp_async16(qa + swz(r, c), a.q + (size_t)(okq ? row0 + r : 0) * kD + c * 8, okq);
    const bool okk = key0 + r < kv_len;
    const size_t off = (size_t)(okk ? key0 + r : 0) * kD + c * 8;
    cp_async16(ka + swz(r, c), kc + off, okk);
    cp_async16(va + swz(r, c), vc + off, okk);
  }
  if (et < kChunk) s_valid[et] = (key0 + et < kv_len && a.key_valid[key0 + et]) ? 1 : 0;
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  named_bar_sync(2, 128);

  const int g = lane >> 2, t4 = lane & 3;
  float s[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
  for (int kk = 0; kk < kD / 16; ++kk) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(qa + swz(wrel * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, kk * 2 + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      uint32_t b0, b1, b2, b3;
      const int mi = lane >> 3;
      ldsm_x4(ka + swz(jj * 16 + (mi >> 1) * 8 + (lane & 7), kk * 2 + (mi & 1)), b0, b1, b2, b3);
      mma_bf16(s[2 * jj], a0, a1, a2, a3, b0, b1);
      mma_bf16(s[2 * jj + 1], a0, a1, a2, a3, b2, b3);
    }
  }
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int key = j * 8 + 2 * t4 + (e & 1);
      float v = bf16_round(bf16_round(s[j][e]) * a.attn_scale);
      v = s_valid[key] ? v : -INFINITY;
      s[j][e] = v;
      mx[e >> 1] = fmaxf(mx[e >> 1], v);
    }
  float ls[2] = {0.f, 0.f};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
    mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2));
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int h = e >> 1;
      const float pv = (s[j][e] == -INFINITY) ? 0.f : __expf(s[j][e] - mx[h]);
      s[j][e] = pv;
      ls[h] += pv;
    }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    ls[h] += __shfl_xor_sync(0xffffffff, ls[h], 1);
    ls[h] += __shfl_xor_sync(0xffffffff, ls[h], 2);
  }
  // O (16 x 256) = P (16 x 64) . V (64 x 256), written straight out as the partial.
#pragma unroll 1
  for (int half = 0; half < 2; ++half) {  // two passes of 16 d-tiles keep registers in check
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
      const uint32_t a0 = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3;
        ldsm_x4_t(va + swz(kk * 16 + (mi & 1) * 8 + (lane & 7), half * 16 + jj * 2 + (mi >> 1)), b0, b1, b2, b3);
        mma_bf16(o[2 * jj], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * jj + 1], a0, a1, a2, a3, b2, b3);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = row0 + wrel * 16 + g + h * 8;
      if (r >= rows) continue;
      float* dst = a.attn_o + ((size_t)sp * rows + r) * kD + half * 128;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        __stcg(reinterpret_cast<float2*>(dst + j * 8 + 2 * t4), make_float2(o[j][2 * h], o[j][2 * h + 1]));
    }
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = row0 + wrel * 16 + g + h * 8;
    if (r < rows && t4 == 0) {
      __stcg(reinterpret_cast<float2*>(a.attn_ml + ((size_t)sp * rows + r) * 2), make_float2(mx[h], ls[h]));
    }
  }
  named_bar_sync(2, 128);  // shared tiles free for the next unit
}

// Combine the split-KV partials of row r (one warp) into attn[r] (bf16).
__device__ void comb_row(const Args& a, int r, int lane) {
  const int rows = a.tokens * a.hq;
  float ms = -INFINITY, lsum = 0.f;
  if (lane < a.attn_splits) {
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.attn_ml + ((size_t)lane * rows + r) * 2));
    ms = ml.x;
    lsum = ml.y;
  }
  float mmax = ms;
  for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffff, mmax, o));
  const float w = (lane < a.attn_splits && ms != -INFINITY) ? __expf(ms - mmax) : 0.f;
  float l = lsum * w;
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffff, l, o);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int s0 = 0; s0 < a.attn_splits; s0 += 4) {
    float4 va[4], vb[4];
    float ws[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int sj = s0 + j;
      ws[j] = __shfl_sync(0xffffffff, w, sj & 31);
      if (sj < a.attn_splits) {
        const float4* src = reinterpret_cast<const float4*>(a.attn_o + ((size_t)sj * rows + r) * kD + lane * 8);
        va[j] = __ldcg(src);
        vb[j] = __ldcg(src + 1);
      } else {
        ws[j] = 0.f;
        va[j] = vb[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[0] += va[j].x * ws[j]; acc[1] += va[j].y * ws[j]; acc[2] += va[j].z * ws[j]; acc[3] += va[j].w * ws[j];
      acc[4] += vb[j].x * ws[j]; acc[5] += vb[j].y * ws[j]; acc[6] += vb[j].z * ws[j]; acc[7] += vb[j].w * ws[j];
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  float o[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = acc[j] * inv;
  *reinterpret_cast<uint4*>(a.attn + (size_t)r * kD + lane * 8) = pack8(o);
}

// GEMM unit epilogue: drain TMEM, publish the split partial, meet the tile's
// other splits, reduce + apply the fused epilogue to this split's slice.
template <int EPI>
__device__ bool gemm_epilogue(const Args& a, int op, const SkinnyParams& p, int iter, uint32_t tmem, int& ucount,
                              uint64_t* tfull, uint64_t* tempty, volatile int* s_abort, int* s_flag, int et, int wq,
                              int lane, int ev) {
  const GemmShape g = a.g[op];
  const int cta = blockIdx.x;
  const int tile = cta / g.splits, split = cta % g.splits;
  const int b = ucount & 1;
  const uint32_t par = (ucount >> 1) & 1;
  ++ucount;
  // One thread makes the bounded wait; the decision is shared so that all 128
  // threads take the same path through the named barriers below.
  if (et == 0) s_flag[2] = mbar_wait_abort(&tfull[b], par, s_abort, a.status, PI05_DEV_TIMEOUT_EPILOGUE) ? 1 : 0;
  named_bar_sync(1, 128);
  if (!s_flag[2]) return false;
  if (et == 0) stamp(a, iter, ev);
  while (!mbar_try_wait(smem_u32(&tfull[b]), par)) {
  }  // phase already complete: returns at once, orders this thread after the MMAs
  tc_fence_after();
  const uint32_t tbase = tmem + b * kTok + ((uint32_t)(wq * 32) << 16);
  const int r = wq * 32 + lane;
  float* part = a.part[op] + ((size_t)tile * g.splits) * kTok * kBM;
  float* mine = part + (size_t)split * kTok * kBM;
  // Publish this split's partial (row r of the tile, all tokens), 32 columns at a time.
#pragma unroll 1
  for (int c = 0; c < kTok / 32; ++c) {
    float v[32];
    tmem_ld32(tbase + c * 32, v);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c * 32 + j < a.tokens) __stcg(mine + (c * 32 + j) * kBM + r, v[j]);
  }
  tc_fence_before();
  named_bar_sync(1, 128);
  if (et == 0) mbar_arrive(&tempty[b]);
  __threadfence();
  named_bar_sync(1, 128);
  if (et == 0) {
    int* cnt = a.tile_cnt + (op * 64 + tile) * kCtrStride;
    atomicAdd(cnt, 1);
    s_flag[0] = wait_geq(cnt, (iter + 1) * g.splits, s_abort, a.status) ? 1 : 0;
  }
  named_bar_sync(1, 128);
  if (!s_flag[0]) return false;
  if (et == 0) stamp(a, iter, ev + 1);
  __threadfence();
  TileSrc src{nullptr, part, g.splits, kTok * kBM};
  const int items = epi_items<EPI>(p, tile, a.tokens);
  const int i0 = (int)(((long)split * items) / g.splits);
  const int i1 = (int)(((long)(split + 1) * items) / g.splits);
  apply_epilogue<EPI, 1>(p, src, tile, 0, i0, i1, et);
  return true;
}

__global__ void __launch_bounds__(kThreads, 1) denoise_mega_kernel(const __grid_constant__ Maps maps,
                                                                    const __grid_constant__ Args a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* sQ = ring + kStages * kStageBytes;
  uint8_t* sK = sQ + 64 * kRowBytes;
  uint8_t* sV = sK + 64 * kRowBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sV + 64 * kRowBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_drain = tempty + 2;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(mma_drain + 1);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  int* s_flag = const_cast<int*>(reinterpret_cast<volatile int*>(s_abort + 1));  // [4]
  float* s_red = reinterpret_cast<float*>(s_flag + 4);  // [8 + 32]
  uint8_t* s_valid = reinterpret_cast<uint8_t*>(s_red + 48);
  float* s_hn = reinterpret_cast<float*>(sQ);           // final rows reuse the attention tiles

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = blockIdx.x, nct = gridDim.x;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 2);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 1);
    }
    mbar_init(mma_drain, 1);
    *s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, 2 * kTok);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const int n_iter = a.num_steps * a.depth;
  const int T = a.tokens;

  if (warp == 0) {
    // ---------------- weight TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      uint32_t seq = 0;
      for (int it = 0; it < n_iter && !abort_set(s_abort); ++it) {
        const int l = it % a.depth;
        for (int op = 0; op < 4; ++op) {
          const GemmShape g = a.g[op];
          if (cta >= g.tiles * g.splits) continue;
          const int tile = cta / g.splits, split = cta % g.splits;
          const int kb0 = (split * g.kb) / g.splits, kb1 = ((split + 1) * g.kb) / g.splits;
          const SkinnyParams p = op_params(a, op, l, a.mod_table);
          const TileRows tr = op_rows(p, op, tile);
          const CUtensorMap* m0 = wmap(maps, l, op, 0);
          const CUtensorMap* m1 = wmap(maps, l, op, 1);
          for (int kb = kb0; kb < kb1; ++kb, ++seq) {
            const int st = seq % kStages;
            if (!mbar_wait_abort(&empty[st], ((seq / kStages) & 1) ^ 1, s_abort, a.status,
                                 PI05_DEV_TIMEOUT_PRODUCER))
              break;
            mbar_arrive_expect_tx(&full[st], kWBytes);
            tma_load_2d(ring + st * kStageBytes, m0, &full[st], kb * kBK, tr.row0, pol);
            tma_load_2d(ring + st * kStageBytes + kWBytes / 2, m1, &full[st], kb * kBK, tr.row1, pol);
          }
        }
      }
    }
  } else if (warp == 2) {
    // ---------------- activation TMA producer ----------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_last();
      uint32_t seq = 0;
      for (int it = 0; it < n_iter && !abort_set(s_abort); ++it) {
        for (int op = 0; op < 4; ++op) {
          const GemmShape g = a.g[op];
          if (cta >= g.tiles * g.splits) continue;
          const int split = cta % g.splits;
          const int kb0 = (split * g.kb) / g.splits, kb1 = ((split + 1) * g.kb) / g.splits;
          // input of this op complete for iteration `it`
          int* ctr;
          int target;
          if (op == OP_QKV) { ctr = a.done + PH_NORM1 * kCtrStride; target = T * (it + 1); }
          else if (op == OP_O) { ctr = a.done + PH_COMB * kCtrStride; target = a.comb_units * (it + 1); }
          else if (op == OP_GU) { ctr = a.done + PH_NORM2 * kCtrStride; target = T * (it + 1); }
          else { ctr = a.done + PH_GEGLU * kCtrStride; target = a.g[OP_GU].tiles * a.g[OP_GU].splits * (it + 1); }
          if (!wait_geq(ctr, target, s_abort, a.status)) break;
          asm volatile("fence.proxy.async.global;" ::: "memory");
          const CUtensorMap* xm = &maps.x[op];
          bool ok = true;
          for (int kb = kb0; kb < kb1; ++kb, ++seq) {
            const int st = seq % kStages;
            if (!mbar_wait_abort(&empty[st], ((seq / kStages) & 1) ^ 1, s_abort, a.status,
                                 PI05_DEV_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[st], kXBytes);
            tma_load_2d(ring + st * kStageBytes + kWBytes, xm, &full[st], kb * kBK, 0, pol);
          }
          if (!ok) break;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = umma_idesc_bf16(kBM, kTok);
      uint32_t seq = 0;
      int ucount = 0;
      bool ok = true;
      for (int it = 0; it < n_iter && ok; ++it) {
        for (int op = 0; op < 4 && ok; ++op) {
          const GemmShape g = a.g[op];
          if (cta >= g.tiles * g.splits) continue;
          const int split = cta % g.splits;
          const int kb0 = (split * g.kb) / g.splits, kb1 = ((split + 1) * g.kb) / g.splits;
          const int b = ucount & 1;
          if (!mbar_wait_abort(&tempty[b], ((ucount >> 1) & 1) ^ 1, s_abort, a.status, PI05_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + b * kTok;
          for (int kb = kb0; kb < kb1; ++kb, ++seq) {
            const int st = seq % kStages;
            if (!mbar_wait_abort(&full[st], (seq / kStages) & 1, s_abort, a.status, PI05_DEV_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(ring + st * kStageBytes);
            const uint32_t b0 = a0 + kWBytes;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_bf16(d, umma_sdesc_sw128(a0 + kk * 32), umma_sdesc_sw128(b0 + kk * 32), kIdesc,
                        (kb > kb0 || kk > 0) ? 1u : 0u);
            umma_commit(&empty[st]);
          }
          if (ok) umma_commit(&tfull[b]);
          ++ucount;
        }
      }
      // all issued MMAs complete before TMEM is released
      umma_commit(mma_drain);
      if (!mbar_wait(mma_drain, 0)) report_status(a.status, PI05_DEV_TIMEOUT_DRAIN);
    }
  } else if (warp >= kWorkerWarp0) {
    // ---------------- workers ----------------
    const int et = threadIdx.x - kWorkerWarp0 * 32;
    const int wrel = warp - kWorkerWarp0;
    const int wq = warp & 3;
    const int row_t = nct - 1 - cta;  // norm / final row owned by this CTA
    int ucount = 0;
    bool ok = true;
    for (int s = 0; s < a.num_steps && ok; ++s) {
      const float* mods = a.mod_table + (size_t)s * a.n_norm * 3 * a.width;
      for (int l = 0; l < a.depth && ok; ++l) {
        const int it = s * a.depth + l;
        // adaRMS 1 (layer 0: action_in_proj first)
        if (row_t < T) {
          if (l > 0) {
            if (et == 0) s_flag[1] = wait_geq(a.done + PH_DOWN * kCtrStride, a.g[OP_DOWN].tiles * a.g[OP_DOWN].splits * it,
                                              s_abort, a.status);
            named_bar_sync(1, 128);
            if (!s_flag[1]) { ok = false; break; }
            __threadfence();
          }
          if (et == 0) stamp(a, it, 0);
          norm_row(a, row_t, l == 0, mods + (size_t)(2 * l) * 3 * a.width, a.xn1, s_red, et, wrel, lane);
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_NORM1 * kCtrStride); stamp(a, it, 1); }
        }
        // q|k|v + RoPE
        if (cta < a.g[OP_QKV].tiles * a.g[OP_QKV].splits) {
          const SkinnyParams p = op_params(a, OP_QKV, l, mods);
          if (!gemm_epilogue<SK_EPI_QKV_ROPE>(a, OP_QKV, p, it, tmem, ucount, tfull, tempty, s_abort, s_flag, et, wq,
                                               lane, 2)) { ok = false; break; }
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_QKV * kCtrStride); stamp(a, it, 4); }
        }
        // attention partials
        const int au = nct - 1 - cta;
        if (au < a.attn_units) {
          if (et == 0) s_flag[1] = wait_geq(a.done + PH_QKV * kCtrStride, a.g[OP_QKV].tiles * a.g[OP_QKV].splits * (it + 1),
                                            s_abort, a.status);
          named_bar_sync(1, 128);
          if (!s_flag[1]) { ok = false; break; }
          __threadfence();
          if (et == 0) stamp(a, it, 5);
          attn_unit(a, l, au, sQ, sK, sV, s_valid, et, wrel, lane);
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_ATTN * kCtrStride); stamp(a, it, 6); }
        }
        // split combine -> attn (bf16)
        const int cu = nct - 1 - cta;
        if (cu < a.comb_units) {
          if (et == 0) s_flag[1] = wait_geq(a.done + PH_ATTN * kCtrStride, a.attn_units * (it + 1), s_abort, a.status);
          named_bar_sync(1, 128);
          if (!s_flag[1]) { ok = false; break; }
          __threadfence();
          if (et == 0) stamp(a, it, 7);
          const int r = cu * 4 + wrel;
          if (r < T * a.hq) comb_row(a, r, lane);
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_COMB * kCtrStride); stamp(a, it, 8); }
        }
        // o_proj + gated residual
        if (cta < a.g[OP_O].tiles * a.g[OP_O].splits) {
          const SkinnyParams p = op_params(a, OP_O, l, mods);
          if (!gemm_epilogue<SK_EPI_GATED_RESID>(a, OP_O, p, it, tmem, ucount, tfull, tempty, s_abort, s_flag, et,
                                                  wq, lane, 9)) { ok = false; break; }
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_OPROJ * kCtrStride); stamp(a, it, 11); }
        }
        // adaRMS 2
        if (row_t < T) {
          if (et == 0) s_flag[1] = wait_geq(a.done + PH_OPROJ * kCtrStride, a.g[OP_O].tiles * a.g[OP_O].splits * (it + 1),
                                            s_abort, a.status);
          named_bar_sync(1, 128);
          if (!s_flag[1]) { ok = false; break; }
          __threadfence();
          if (et == 0) stamp(a, it, 12);
          norm_row(a, row_t, false, mods + (size_t)(2 * l + 1) * 3 * a.width, a.xn2, s_red, et, wrel, lane);
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_NORM2 * kCtrStride); stamp(a, it, 13); }
        }
        // gate/up + GeGLU
        if (cta < a.g[OP_GU].tiles * a.g[OP_GU].splits) {
          const SkinnyParams p = op_params(a, OP_GU, l, mods);
          if (!gemm_epilogue<SK_EPI_GEGLU>(a, OP_GU, p, it, tmem, ucount, tfull, tempty, s_abort, s_flag, et, wq,
                                            lane, 14)) { ok = false; break; }
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_GEGLU * kCtrStride); stamp(a, it, 16); }
        }
        // down + gated residual
        if (cta < a.g[OP_DOWN].tiles * a.g[OP_DOWN].splits) {
          const SkinnyParams p = op_params(a, OP_DOWN, l, mods);
          if (!gemm_epilogue<SK_EPI_GATED_RESID>(a, OP_DOWN, p, it, tmem, ucount, tfull, tempty, s_abort, s_flag,
                                                  et, wq, lane, 17)) { ok = false; break; }
          __threadfence();
          named_bar_sync(1, 128);
          if (et == 0) { signal(a.done + PH_DOWN * kCtrStride); stamp(a, it, 19); }
        }
      }
      if (!ok) break;
      // final adaRMS + action_out_proj + Euler
      if (row_t < T) {
        if (et == 0) s_flag[1] = wait_geq(a.done + PH_DOWN * kCtrStride,
                                          a.g[OP_DOWN].tiles * a.g[OP_DOWN].splits * (s + 1) * a.depth, s_abort,
                                          a.status);
        named_bar_sync(1, 128);
        if (!s_flag[1]) { ok = false; break; }
        __threadfence();
        final_row(a, row_t, mods + (size_t)(2 * a.depth) * 3 * a.width, a.ts[s], a.ts[s] - a.ts[s + 1], s_hn,
                  s_red, et, wrel, lane);
        __threadfence();
        named_bar_sync(1, 128);
        if (et == 0) { signal(a.done + PH_FINAL * kCtrStride); if (a.trace) a.trace[(size_t)blockIdx.x * kTraceSlots + kTraceSlots - 64 + s] = globaltimer_ns(); }
      }
    }
    if (!ok && et == 0) *s_abort = 1;
  }

  // ---------------- teardown ----------------
  __syncwarp();
  __syncthreads();
  if (abort_set(s_abort) && threadIdx.x == 0) {
    // let any TMA copies still in flight land before shared memory is released
    const uint64_t t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < 200000ull) {
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kTok);
  }
}

}  // namespace mega
}  // namespace pi05

using namespace pi05;
using namespace pi05::mega;

extern "C" int pi05_trace_slots(void) { return kTraceSlots; }

extern "C" int pi05_denoise_loop_persistent(const Pi05ExpertPlan* P, void* stream) {
  if (P == nullptr || P->layers == nullptr || P->host_timesteps == nullptr || P->mod_table == nullptr) {
    set_last_error("denoise_loop_persistent: null plan field");
    return PI05_ERR_INVALID_ARG;
  }
  const int T = P->tokens, W = P->width, F = P->mlp_dim, HQ = P->n_q_heads, D = P->head_dim;
  if (P->depth > kMaxLayers || P->depth <= 0 || W != 1024 || F % 64 || HQ * D % 64 || D != 256 ||
      P->n_kv_heads != 1 || T > kTok || T <= 0 || P->num_steps > 16 || P->num_steps <= 0 || P->action_dim > 32 ||
      P->kv_rows < P->prefix_len + T) {
    set_last_error("denoise_loop_persistent: unsupported shape (depth=%d width=%d tokens=%d steps=%d)", P->depth, W,
                   T, P->num_steps);
    return PI05_ERR_SHAPE;
  }
  Workspace ws;
  if (split_workspace(P->workspace, P->workspace_bytes, &ws)) {
    set_last_error("denoise_loop_persistent: workspace missing or too small");
    return PI05_ERR_WORKSPACE;
  }
  int dev = 0, sms = 0, coop = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev);
  Args a;
  std::memset(&a, 0, sizeof(a));
  a.depth = P->depth;
  a.width = W;
  a.mlp = F;
  a.hq = HQ;
  a.hd = D;
  a.tokens = T;
  a.action_dim = P->action_dim;
  a.prefix_len = P->prefix_len;
  a.kv_rows = P->kv_rows;
  a.num_steps = P->num_steps;
  a.n_norm = 2 * P->depth + 1;
  a.eps = P->eps;
  a.attn_scale = 1.0f / std::sqrt((float)D);
  // split choices: one unit per CTA per GEMM phase
  const int qkv_tiles = (HQ + 1) * (D / 128) + D / 128;
  a.g[OP_QKV] = {qkv_tiles, std::max(1, std::min(W / 64, sms / qkv_tiles)), W / 64};
  a.g[OP_O] = {W / 128, std::max(1, std::min(HQ * D / 64, sms / (W / 128))), HQ * D / 64};
  a.g[OP_GU] = {F / 64, std::max(1, std::min(W / 64, sms / (F / 64))), W / 64};
  a.g[OP_DOWN] = {W / 128, std::max(1, std::min(F / 64, sms / (W / 128))), F / 64};
  const int rows = T * HQ;
  const int row_blocks = (rows + 63) / 64;
  const int kv_len = P->prefix_len + T;
  a.attn_splits = (kv_len + kChunk - 1) / kChunk;
  a.attn_units = row_blocks * a.attn_splits;
  a.comb_units = (rows + 3) / 4;
  int max_units = std::max(a.attn_units, a.comb_units);
  for (int op = 0; op < 4; ++op) max_units = std::max(max_units, a.g[op].tiles * a.g[op].splits);
  if (!coop || max_units > sms || a.attn_splits > 32 || T > sms || 4 * 64 > 1024) {
    set_last_error("denoise_loop_persistent: needs cooperative launch and >= %d SMs (have %d), <= 32 KV chunks",
                   max_units, sms);
    return PI05_ERR_SHAPE;
  }
  a.h = static_cast<__nv_bfloat16*>(P->h);
  a.xn1 = static_cast<__nv_bfloat16*>(P->xn);
  a.q = static_cast<__nv_bfloat16*>(P->q);
  a.attn = static_cast<__nv_bfloat16*>(P->attn);
  a.act = static_cast<__nv_bfloat16*>(P->act);
  a.rope_cos = static_cast<const __nv_bfloat16*>(P->rope_cos);
  a.rope_sin = static_cast<const __nv_bfloat16*>(P->rope_sin);
  for (int l = 0; l < P->depth; ++l) {
    a.k_cache[l] = static_cast<__nv_bfloat16*>(P->layers[l].k_cache);
    a.v_cache[l] = static_cast<__nv_bfloat16*>(P->layers[l].v_cache);
  }
  a.key_valid = P->key_valid;
  a.mod_table = P->mod_table;
  a.w_in = P->w_in;
  a.b_in = P->b_in;
  a.w_out = P->w_out;
  a.b_out = P->b_out;
  a.x_t = P->x_t;
  a.v_t = P->v_t;
  for (int s = 0; s <= P->num_steps; ++s) a.ts[s] = P->host_timesteps[s];
  // workspace: counters at the top of the counter block (the standalone GEMMs use
  // the bottom), partials in the split-K region, attention partials in scratch.
  // counters: one 128-byte line each, at the start of the scratch region
  const size_t ctr_ints = (size_t)(16 + 4 * 64) * kCtrStride;
  a.done = reinterpret_cast<int*>(ws.scratch);
  a.tile_cnt = a.done + 16 * kCtrStride;
  float* scratch = ws.scratch + ctr_ints;  // 128-byte aligned
  a.trace = P->trace;
  size_t off = 0;
  for (int op = 0; op < 4; ++op) {
    a.part[op] = ws.accum + off / sizeof(float);
    off += (size_t)a.g[op].tiles * a.g[op].splits * kTok * kBM * sizeof(float);
  }
  const size_t attn_bytes = (size_t)a.attn_splits * rows * (kD + 2) * sizeof(float);
  // The second normalised-activation buffer lives in scratch too (xn2 [T, W] bf16).
  const size_t xn2_bytes = (size_t)T * W * 2;
  if (off > ws.accum_bytes || ctr_ints * 4 + attn_bytes + xn2_bytes + 256 > ws.scratch_bytes) {
    set_last_error("denoise_loop_persistent: workspace too small");
    return PI05_ERR_WORKSPACE;
  }
  a.attn_o = scratch;
  a.attn_ml = scratch + (size_t)a.attn_splits * rows * kD;
  a.xn2 = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(scratch) + ((attn_bytes + 255) & ~size_t(255)));
  a.status = ws.status;

  static Maps maps;  // host staging of the tensor maps (passed by value)
  static std::mutex maps_mu;
  std::lock_guard<std::mutex> lock(maps_mu);
  std::memset(&maps, 0, sizeof(maps));
  const int qkv_rows = (HQ + 2) * D;
  for (int l = 0; l < P->depth; ++l) {
    const Pi05ExpertLayer& L = P->layers[l];
    int rc = make_tmap_bf16_2d(&maps.w[l][0], L.w_qkv, qkv_rows, W, W, 64, 64, true);
    if (!rc) rc = make_tmap_bf16_2d(&maps.w[l][1], L.w_o, W, HQ * D, HQ * D, 64, 64, true);
    if (!rc) rc = make_tmap_bf16_2d(&maps.w[l][2], L.w_gate, F, W, W, 64, 64, true);
    if (!rc) rc = make_tmap_bf16_2d(&maps.w[l][3], L.w_up, F, W, W, 64, 64, true);
    if (!rc) rc = make_tmap_bf16_2d(&maps.w[l][4], L.w_down, W, F, F, 64, 64, true);
    if (rc) return rc;
  }
  int rc = make_tmap_bf16_2d(&maps.x[0], a.xn1, T, W, W, kTok, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&maps.x[1], a.attn, T, HQ * D, HQ * D, kTok, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&maps.x[2], a.xn2, T, W, W, kTok, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&maps.x[3], a.act, T, F, F, kTok, 64, true);
  if (rc) return rc;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(a.done, 0, ctr_ints * sizeof(int), st);
  if (e != cudaSuccess) {
    set_last_error("denoise_loop_persistent: counter reset failed: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  const size_t smem = 1024 + kStages * kStageBytes + kAttnSmem + 512;
  static bool attr_done[16] = {false};
  if (dev < 16 && !attr_done[dev]) {
    e = cudaFuncSetAttribute(denoise_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_last_error("denoise_loop_persistent: smem attribute: %s", cudaGetErrorString(e));
      return PI05_ERR_LAUNCH;
    }
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, denoise_mega_kernel, maps, a);
  count_launch();
  if (e != cudaSuccess) {
    set_last_error("denoise_loop_persistent: launch failed: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  return PI05_OK;
}
