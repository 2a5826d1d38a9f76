// SigLIP bidirectional attention (16 heads x head_dim 72, 256 tokens per view) on
// the 5th-generation tensor cores (tcgen05).
//
// A CTA owns 128 query rows of one (view, head) and all 256 keys of that view, so
// the softmax sees whole rows and needs no running max:
//
//   S  = Q . K^T        tcgen05.mma M=128 N=256, K = 80 (head_dim 72 padded by one
//                       16-wide step) -> TMEM columns 0..255
//   P  = softmax(bf16(bf16(S) * scale)) in fp32, cast to bf16   (eager SiglipAttention)
//   O  = P . V          tcgen05.mma M=128 N=80 (dims 72..79 ignored), K = 256 keys
//                       -> TMEM columns 256..335
//
// Operands by TMA with the 128-byte swizzle straight from the q|k|v projection
// output [views*256, 3*1152]: a head's 72 dims are loaded as two 64-wide boxes at
// columns h*72 and h*72+64, so the second box also holds 56 columns of whatever
// follows (the next head, or zero fill past the row).  Only its first 16 columns
// enter an MMA: Q's dims 72..79 are zeroed in shared memory, which cancels K's
// columns there in S; V's extra columns only reach output columns 72..79, which are
// not stored.  P overwrites K's buffer once S is done.
//
// Warp roles: warp 0 TMA, warp 1 TMEM owner + MMA issuer, warps 2-9 softmax and
// output (two per TMEM lane quarter, each owning 128 of a row's 256 keys; the pair
// agrees on the row max and sum through shared memory).
//
// Reference: transformers SiglipAttention (eager), as called by
// pi05_infer/openpi_patched/gemma_pytorch.py:106-107.
#include <cuda_bf16.h>
#include <stdint.h>

#include <cmath>
#include <cstdlib>
#include <cstring>

#include "host_util.h"
#include "ptx.cuh"

namespace pi05 {
namespace {

constexpr int kSeq = 256;                 // tokens per view = keys per row
constexpr int kHd = 72;                   // head dim
constexpr int kRows = 128;                // query rows per CTA (UMMA M)
constexpr int kThreads = 320;             // warp 0 TMA, warp 1 MMA, warps 2-9 softmax / output
constexpr int kSoft = 256;                // softmax threads
constexpr int kQBox = kRows * 128;        // [128 rows x 64 dims] bf16, 16 KB
constexpr int kKBox = kSeq * 128;         // [256 keys x 64 dims] bf16, 32 KB
constexpr int kPBox = kRows * 128;        // [128 rows x 64 keys] bf16, 16 KB
constexpr uint32_t kTmemCols = 512;       // S at 0..255, O at 256..335
constexpr uint32_t kColO = 256;
constexpr uint32_t kIdescS = umma_idesc_bf16(kRows, kSeq);
constexpr uint32_t kIdescPV = umma_idesc_bf16(kRows, 80) | (1u << 16);  // B (V) MN-major

struct SaMaps {
  CUtensorMap q;   // box [128 rows x 64 cols]
  CUtensorMap kv;  // box [256 rows x 64 cols]
};

// Shared memory: Q (2 boxes, 32 KB), K (2 boxes, 64 KB; P's 4 boxes overwrite it
// once S is done), V (2 boxes, 64 KB), barriers and the row-max / row-sum exchange.
constexpr size_t kSmemBytes = 1024 + 2 * kQBox + 2 * kKBox + 2 * kKBox + 16 * 8 + 4 * kRows * 4;

__device__ __forceinline__ uint32_t sw_off(int r, int g) { return (uint32_t)(r * 128 + ((g ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(kThreads, 1)
    siglip_attn_tc_kernel(const __grid_constant__ SaMaps mp, __nv_bfloat16* __restrict__ out, int width, int heads,
                          float scale, int* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                 // 2 x [128 x 64]
  uint8_t* sK = sQ + 2 * kQBox;       // 2 x [256 x 64]; then P: 4 x [128 x 64 keys]
  uint8_t* sV = sK + 2 * kKBox;       // 2 x [256 x 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * kKBox);
  uint64_t* q_full = bars;            // Q landed
  uint64_t* k_full = bars + 1;        // K landed
  uint64_t* v_full = bars + 2;        // V landed
  uint64_t* s_full = bars + 3;        // S in TMEM
  uint64_t* p_full = bars + 4;        // P written (256 arrivals)
  uint64_t* o_full = bars + 5;        // O in TMEM
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 6);
  float* s_red = reinterpret_cast<float*>(bars + 16);  // [2 halves][128 rows] max, then [2][128] sums

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int vh = blockIdx.x, view = vh / heads, h = vh - view * heads;
  const int q0 = blockIdx.y * kRows;
  const int row_base = view * kSeq;  // first token of the view
  const int xq = h * kHd, xk = width + h * kHd, xv = 2 * width + h * kHd;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(k_full, 1);
    mbar_init(v_full, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, kSoft);
    mbar_init(o_full, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&mp.q);
    prefetch_tmap(&mp.kv);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();
      const uint64_t pol = l2_policy_evict_first();
      mbar_arrive_expect_tx(q_full, 2 * kQBox);
      for (int b = 0; b < 2; ++b) tma_load_2d(sQ + b * kQBox, &mp.q, q_full, xq + b * 64, row_base + q0, pol);
      mbar_arrive_expect_tx(k_full, 2 * kKBox);
      for (int b = 0; b < 2; ++b) tma_load_2d(sK + b * kKBox, &mp.kv, k_full, xk + b * 64, row_base, pol);
      mbar_arrive_expect_tx(v_full, 2 * kKBox);
      for (int b = 0; b < 2; ++b) tma_load_2d(sV + b * kKBox, &mp.kv, v_full, xv + b * 64, row_base, pol);
    }
  } else if (warp == 1) {
    bool ok = mbar_wait(q_full, 0);
    // Q's dims 72..79 (16-byte chunk 1 of the second box) are zero, so K's columns
    // there add nothing to S.
    if (ok)
      for (int r = lane; r < kRows; r += 32)
        *reinterpret_cast<uint4*>(sQ + kQBox + sw_off(r, 1)) = make_uint4(0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      ok = ok && mbar_wait(k_full, 0);
      if (ok) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(sQ), b0 = smem_u32(sK);
        // dims 0..63 (4 steps of 16), then dims 64..79 (one step)
#pragma unroll
        for (int kk = 0; kk < 5; ++kk) {
          const int b = kk >> 2, k16 = kk & 3;
          umma_bf16(tmem, umma_sdesc_sw128(a0 + b * kQBox + k16 * 32), umma_sdesc_sw128(b0 + b * kKBox + k16 * 32),
                    kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
      }
      ok = ok && mbar_wait(p_full, 0) && mbar_wait(v_full, 0);
      if (ok) {
        tc_fence_after();
        const uint32_t a0 = smem_u32(sK), b0 = smem_u32(sV);
        // 16 steps of 16 keys: P box kk / 4, V rows kk*16 .. (MN-major, the two
        // 64-dim boxes 32 KB apart)
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          umma_bf16(tmem + kColO, umma_sdesc_sw128(a0 + (kk >> 2) * kPBox + (kk & 3) * 32),
                    umma_sdesc_mn_sw128(b0 + kk * 2048, kKBox, 1024), kIdescPV, kk > 0 ? 1u : 0u);
        umma_commit(o_full);
      } else {
        report_status(status, PI05_DEV_TIMEOUT_MMA);
      }
    }
  } else {
    // Softmax warps 2..9: TMEM lane quarter q = warp % 4 (rows q*32 .. q*32+31, one
    // per thread); half hh takes keys hh*128 .. hh*128+127 of the row.
    const int q = warp & 3;
    const int hh = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    bool ok = mbar_wait(s_full, 0);
    tc_fence_after();
    float sv[128];
    float mx = -INFINITY;
    if (ok) {
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + hh * 128 + c * 32, sv + c * 32);
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        // bf16(bf16(q.k) * scale), two values per conversion
        bf16_round2(sv[i], sv[i + 1]);
        sv[i] *= scale;
        sv[i + 1] *= scale;
        bf16_round2(sv[i], sv[i + 1]);
        mx = fmaxf(mx, fmaxf(sv[i], sv[i + 1]));
      }
    }
    s_red[hh * kRows + r] = mx;
    named_bar_sync(1 + q, 64);
    const float m = fmaxf(s_red[r], s_red[kRows + r]);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 128; ++i) {
      sv[i] = __expf(sv[i] - m);
      sum += sv[i];
    }
    s_red[2 * kRows + hh * kRows + r] = sum;
    named_bar_sync(1 + q, 64);
    const float lsum = s_red[2 * kRows + r] + s_red[3 * kRows + r];  // half 0 + half 1
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    // P = bf16(e / sum) into the K buffer (K-major, 128-byte swizzle, 64 keys a box).
    uint8_t* sP = sK;
#pragma unroll
    for (int g8 = 0; g8 < 16; ++g8) {
      const int key = hh * 128 + g8 * 8;
      uint4 u;
      u.x = pack_bf16x2(sv[g8 * 8 + 0] * inv, sv[g8 * 8 + 1] * inv);
      u.y = pack_bf16x2(sv[g8 * 8 + 2] * inv, sv[g8 * 8 + 3] * inv);
      u.z = pack_bf16x2(sv[g8 * 8 + 4] * inv, sv[g8 * 8 + 5] * inv);
      u.w = pack_bf16x2(sv[g8 * 8 + 6] * inv, sv[g8 * 8 + 7] * inv);
      *reinterpret_cast<uint4*>(sP + (key >> 6) * kPBox + sw_off(r, (key & 63) >> 3)) = u;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(p_full);
    ok = ok && mbar_wait(o_full, 0);
    if (!ok) report_status(status, PI05_DEV_TIMEOUT_EPILOGUE);
    tc_fence_after();
    if (ok) {
      // O columns: half 0 stores dims 0..31 and 64..71, half 1 dims 32..63.
      __nv_bfloat16* dst = out + (size_t)(row_base + q0 + r) * width + h * kHd;
      float o[32];
      tmem_ld32(tmem + lane_base + kColO + hh * 32, o);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 u;
        u.x = pack_bf16x2(o[g * 8 + 0], o[g * 8 + 1]);
        u.y = pack_bf16x2(o[g * 8 + 2], o[g * 8 + 3]);
        u.z = pack_bf16x2(o[g * 8 + 4], o[g * 8 + 5]);
        u.w = pack_bf16x2(o[g * 8 + 6], o[g * 8 + 7]);
        *reinterpret_cast<uint4*>(dst + hh * 32 + g * 8) = u;
      }
      if (hh == 0) {
        tmem_ld32(tmem + lane_base + kColO + 64, o);
        uint4 u;
        u.x = pack_bf16x2(o[0], o[1]);
        u.y = pack_bf16x2(o[2], o[3]);
        u.z = pack_bf16x2(o[4], o[5]);
        u.w = pack_bf16x2(o[6], o[7]);
        *reinterpret_cast<uint4*>(dst + 64) = u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

int siglip_attention_tc_run(const void* qkv, int views, int width, int heads, void* out, int* status,
                            cudaStream_t stream) {
  SaMaps mp;
  std::memset(&mp, 0, sizeof(mp));
  const uint64_t rows = (uint64_t)views * kSeq, cols = 3ull * width;
  int rc = make_tmap_bf16_2d(&mp.q, qkv, rows, cols, cols, kRows, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&mp.kv, qkv, rows, cols, cols, kSeq, 64, true);
  if (rc) return rc;
  static bool attr_done[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_done[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(siglip_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) {
      set_last_error("siglip attention smem attr: %s", cudaGetErrorString(e));
      return PI05_ERR_LAUNCH;
    }
    attr_done[dev] = true;
  }
  return launch_pdl(siglip_attn_tc_kernel, dim3(views * heads, kSeq / kRows), dim3(kThreads), kSmemBytes, stream,
                    pdl_enabled(), mp, static_cast<__nv_bfloat16*>(out), width, heads,
                    1.0f / std::sqrt((float)kHd), status);
}

}  // namespace pi05
