// Multi-query flash attention on the 5th-generation tensor cores (tcgen05).
//
// All query heads share the single KV head, so the query rows (token, head) form
// one [R, 256] matrix; a CTA owns 128 query rows and a contiguous range of
// 64-key chunks (split-KV across CTAs when the row blocks alone do not fill the
// GPU).  Per chunk j:
//
//   S_j  = Q . K_j^T          tcgen05.mma M=128 N=64  K=256 -> TMEM (two S buffers)
//   P_j  = exp(S_j - m)       two threads per query row (one per 32-key half) read
//                             the row's S from TMEM, agree on the row max through
//                             shared memory, keep partial row sums, rescale their
//                             half of the O row in TMEM when the exponent base
//                             moved, and write P_j (bf16) to shared memory in the
//                             128B-swizzled K-major layout
//   O   += P_j . V_j          tcgen05.mma M=128 N=256 K=64, V read MN-major straight
//                             from the cache layout [key][256]
//
// Warp roles: warp 0 TMA (Q once, K and V chunks through 1- or 2-stage rings, a
// K slot released after its S, a V slot after its P.V),
// warp 1 TMEM owner + MMA issuer (S_{j+1} is issued before P_j is ready, so the
// tensor core works on the next scores while the softmax runs), warps 2-9
// softmax and the output (two per TMEM lane quarter, so every SM sub-partition
// runs two of them).  Chunks of the static part of the cache (the prefix rows) are
// loaded before the grid-dependency wait; the key mask of the CTA's keys is staged
// in shared memory once.
//
// Numerics follow eager_attention_forward (pi05_infer/gemma/modeling_gemma.py:
// 252-275) the same way as the mma.sync kernel in attention.cu: the score is the
// bf16-rounded Q.K^T times the scale rounded again to bf16, masked keys are
// excluded, softmax in fp32 with a running max, probabilities enter P.V as bf16,
// fp32 accumulation.  The exponent base is the running max held back by up to 8
// (lazy rescaling), which changes no normalised value.  Split-KV partials use the
// mma.sync kernel's layout; two splits merge inside this kernel (the row block's two
// split CTAs form a cluster and exchange halves of O through distributed shared
// memory), more go through the combine kernel.
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "attention.h"
#include "host_util.h"
#include "ptx.cuh"

namespace pi05 {
namespace {

constexpr int kD = 256;
constexpr int kBR = 128;                     // query rows per CTA (UMMA M)
constexpr int kBC = 64;                      // keys per chunk
constexpr int kQBytes = kBR * kD * 2;        // 4 boxes of [128 rows x 64 dims]
constexpr int kKVBytes = kBC * kD * 2;       // 4 boxes of [64 keys x 64 dims]
constexpr int kPBytes = kBR * kBC * 2;       // [128 rows x 64 keys]
constexpr int kThreads = 320;       // warp 0 TMA, warp 1 MMA, warps 2-9 softmax / output
constexpr int kSoftThreads = 256;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 128;              // S buffers at columns 0 and 64, O at 128..383
constexpr uint32_t kIdescS = umma_idesc_bf16(kBR, kBC);
constexpr uint32_t kIdescPV = umma_idesc_bf16(kBR, kD) | (1u << 16);  // B (V) MN-major

// out: bf16 [R, 256] output (no split); po: fp32 split partials [splits * part_rows, 256].
struct TcMaps {
  CUtensorMap q, k, v, out, po;
};

constexpr int kMaxChunks = 64;  // key chunks per CTA whose mask bytes are staged (4096 keys)
constexpr uint32_t kMrgRowBytes = 32 * 128 * 4;  // split merge: a lane quarter's rows of one O half (fp32)
constexpr uint32_t kMrgMlBytes = 32 * 2 * 4;     // and their (m, l) pairs
// Ring, barriers, the row-max / row-sum exchange [6][128], the staged key mask.
size_t tc_smem_bytes(int nst) {
  return 1024 + kQBytes + (size_t)nst * 2 * kKVBytes + kPBytes + 44 * 8 + 6 * kBR * 4 + kMaxChunks * kBC;
}

__device__ __forceinline__ uint32_t p_off(int r, int g) { return (uint32_t)(r * 128 + ((g ^ (r & 7)) << 4)); }

// 32-bit word wd (bytes 4wd .. 4wd+3) of a 32-byte key mask held in two uint4.
__device__ __forceinline__ uint32_t& mask_word(uint4* vk, int wd) { return (&vk[wd >> 2].x)[wd & 3]; }

__device__ __forceinline__ bool key_ok(uint4* vk, int i) { return ((mask_word(vk, i >> 2) >> ((i & 3) * 8)) & 0xffu) != 0; }

__device__ __forceinline__ bool has_zero_byte(uint32_t w) { return ((w - 0x01010101u) & ~w & 0x80808080u) != 0; }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(kThreads, 1) mqa_tc_kernel(const __grid_constant__ TcMaps mp, const AttnParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int nst = p.nbuf;
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kQBytes;
  uint8_t* sV = sK + nst * kKVBytes;
  uint8_t* sP = sV + nst * kKVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kPBytes);
  uint64_t* q_full = bars;        // Q landed
  uint64_t* k_full = bars + 1;    // [2] K chunk landed
  uint64_t* k_empty = bars + 3;   // [2] S of the chunk done (its K slot is free)
  uint64_t* s_full = bars + 5;    // [2] S buffer written
  uint64_t* s_empty = bars + 7;   // [2] S buffer read (128 arrivals)
  uint64_t* p_full = bars + 9;    // P written, O rescaled (128 arrivals)
  uint64_t* p_empty = bars + 10;  // P.V done (P free, O stable)
  uint64_t* mdone = bars + 11;    // every MMA of the CTA complete
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 12);
  int* s_flag = reinterpret_cast<int*>(s_tmem + 1);  // [0] abort, [1] K chunks armed, [2] V chunks armed
  // Per S parity, half and TMEM lane quarter: whether the warp's waits all succeeded
  // (read by the quarter's other warp after their named barrier).
  int* s_pair_ok = reinterpret_cast<int*>(bars + 14);  // [2][2][4]
  uint64_t* lbar = bars + 22;  // [4] row sums, [4] mask staged
  uint64_t* v_full = bars + 28;   // [2] V chunk landed
  uint64_t* v_empty = bars + 30;  // [2] P.V of the chunk done (its V slot is free)
  uint64_t* rfree = bars + 32;   // split merge: the peer CTA's rings are free (one remote arrival)
  uint64_t* rrecv = bars + 34;   // [4] split merge: the peer's rows of a lane quarter landed
  // Row max of each half for the two S parities [2][2][128], then the row sums [2][128].
  float* s_red = reinterpret_cast<float*>(bars + 44);
  uint8_t* s_mask = reinterpret_cast<uint8_t*>(s_red + 6 * kBR);  // [nc * 64] key-mask bytes of this CTA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tr = p.trace != nullptr && threadIdx.x == 64;
  const uint64_t t_entry = tr ? globaltimer_ns() : 0;
  uint64_t t_wait = 0, t_data = 0, t_loop = 0;
  const int row0 = blockIdx.x * kBR;
  const int split = blockIdx.y;
  const int n_chunks_total = (p.kv_len + kBC - 1) / kBC;
  const int c_begin = (split * n_chunks_total) / p.splits;
  const int c_end = ((split + 1) * n_chunks_total) / p.splits;
  const int nc = c_end - c_begin;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kSoftThreads);
    }
    mbar_init(p_full, kSoftThreads);
    mbar_init(p_empty, 1);
    mbar_init(mdone, 1);
    mbar_init(&lbar[4], kSoftThreads);  // mask bytes staged
    mbar_init(rfree, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&rrecv[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&lbar[i], 64);
    s_flag[0] = 0;
    s_flag[1] = 0;
    s_flag[2] = 0;
    fence_mbar_init();
    // Split merge: each lane quarter receives the peer's 32 rows x 128 fp32 columns
    // and their (m, l) pairs.
    if (p.cluster_merge)
      for (int i = 0; i < 4; ++i) mbar_arrive_expect_tx(&rrecv[i], kMrgRowBytes + kMrgMlBytes);
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&mp.q);
    prefetch_tmap(&mp.k);
    prefetch_tmap(&mp.v);
    prefetch_tmap(p.splits == 1 ? &mp.out : &mp.po);
    if (p.cluster_merge) prefetch_tmap(&mp.out);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  // Split merge: both CTAs' barriers are initialised and armed before either
  // signals or copies into the other.
  if (p.cluster_merge) {
    cluster_arrive_release();
    cluster_wait();
  }
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_kv = l2_policy_evict_last();
      int armed_k = 0, armed_v = 0;
      // K and V of a chunk use separate slots: chunk j's K slot is free once S_j is
      // done, its V slot once P_j.V_j is, so K_{j+nst} streams in while the
      // softmax of chunk j still runs.
      auto load_half = [&](int j, bool is_v) -> bool {
        const int st = j % nst;
        uint64_t* full = is_v ? v_full : k_full;
        uint64_t* empty = is_v ? v_empty : k_empty;
        if (j >= nst && !mbar_wait(&empty[st], ((j / nst) - 1) & 1)) {
          report_status(p.status, PI05_DEV_TIMEOUT_PRODUCER);
          s_flag[0] = 1;
          return false;
        }
        mbar_arrive_expect_tx(&full[st], kKVBytes);
        const int key0 = (c_begin + j) * kBC;
        uint8_t* dst = (is_v ? sV : sK) + st * kKVBytes;
        for (int b = 0; b < 4; ++b) tma_load_2d(dst + b * 8192, is_v ? &mp.v : &mp.k, &full[st], b * 64, key0, pol_kv);
        ++(is_v ? armed_v : armed_k);
        return true;
      };
      auto load_kv = [&](int j) -> bool { return load_half(j, false) && load_half(j, true); };
      // Chunk 0 from the static rows does not depend on the previous kernel.
      const bool first_static = nc > 0 && (c_begin + 1) * kBC <= p.static_rows;
      if (first_static) load_kv(0);
      pdl_wait();
      mbar_arrive_expect_tx(q_full, kQBytes);
      for (int b = 0; b < 4; ++b) tma_load_2d(sQ + b * 16384, &mp.q, q_full, b * 64, row0, l2_policy_evict_first());
      bool ok = true;
      if (!first_static && nc > 0) ok = load_kv(0);
      for (int j = 1; j < nc && ok; ++j) ok = load_kv(j);
      s_flag[1] = armed_k;
      s_flag[2] = armed_v;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0);
      auto issue_s = [&](int j) -> bool {
        const int st = j % nst, sb = j & 1;
        if (!mbar_wait(&k_full[st], (j / nst) & 1)) return false;
        if (j >= 2 && !mbar_wait(&s_empty[sb], ((j >> 1) - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(sb * kBC);
        const uint32_t a0 = smem_u32(sQ), b0 = smem_u32(sK + st * kKVBytes);
#pragma unroll
        for (int b = 0; b < 4; ++b)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(d, umma_sdesc_sw128(a0 + b * 16384 + kk * 32), umma_sdesc_sw128(b0 + b * 8192 + kk * 32),
                      kIdescS, (b | kk) ? 1u : 0u);
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
        return true;
      };
      if (ok && nc > 0) ok = issue_s(0);
      for (int j = 0; j < nc && ok; ++j) {
        if (j + 1 < nc) ok = issue_s(j + 1);
        const int st = j % nst;
        if (!ok || !mbar_wait(p_full, j & 1) || !mbar_wait(&v_full[st], (j / nst) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sP), b0 = smem_u32(sV + st * kKVBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tmem + kColO, umma_sdesc_sw128(a0 + kk * 32), umma_sdesc_mn_sw128(b0 + kk * 2048, 8192, 1024),
                    kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(p_empty);
        umma_commit(&v_empty[st]);
      }
      if (!ok) {
        report_status(p.status, PI05_DEV_TIMEOUT_MMA);
        s_flag[0] = 1;
      }
      umma_commit(mdone);
      if (!mbar_wait(mdone, 0)) report_status(p.status, PI05_DEV_TIMEOUT_DRAIN);
    }
  } else {
    // Softmax warps 2..9: TMEM lane quarter = warp % 4 (rows q*32 .. q*32+31, one
    // per thread).  The quarter's two warps split the chunk's 64 score columns
    // (half hh takes keys hh*32 .. hh*32+31) and the 256 O columns (hh*128 ..
    // hh*128+127): they agree on the row max through shared memory once per chunk
    // and keep partial row sums, added at the end.  Two warps per SM sub-partition
    // hide each other's latencies.
    pdl_wait();
    if (tr) t_wait = globaltimer_ns();
    const int q = warp & 3;
    const int hh = (warp - 2) >> 2;
    const int r = q * 32 + lane;
    const int grow = row0 + r;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;

    bool ok = true;
    {
      // Stage this CTA's key-mask bytes (0 past kv_len) once: four per thread.
      const int et = threadIdx.x - 64;
      const int kbeg = c_begin * kBC;
      for (int i = et * 4; i < nc * kBC; i += kSoftThreads * 4) {
        uint32_t word = 0;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int key = kbeg + i + b;
          if (key < p.kv_len && p.key_valid[key] != 0) word |= 1u << (8 * b);
        }
        *reinterpret_cast<uint32_t*>(s_mask + i) = word;
      }
      mbar_arrive(&lbar[4]);
      if (!mbar_wait(&lbar[4], 0)) ok = false;
    }
    float m = -INFINITY, l = 0.f;
    constexpr float kLog2e = 1.4426950408889634f;
    int sexp;
    const bool scale_pow2 = frexpf(p.scale, &sexp) == 0.5f;
    for (int j = 0; j < nc; ++j) {
      const int sb = j & 1;
      // This half's 32 key-mask bytes.
      uint4 vk[2];
      vk[0] = *reinterpret_cast<const uint4*>(s_mask + j * kBC + hh * 32);
      vk[1] = *reinterpret_cast<const uint4*>(s_mask + j * kBC + hh * 32 + 16);
      bool all_valid = true;
#pragma unroll
      for (int wd = 0; wd < 8; ++wd) all_valid = all_valid && !has_zero_byte(mask_word(vk, wd));
      // A failed wait does not leave the loop before the pair's exchange below:
      // both warps of the quarter leave together there (a named barrier).
      if (ok && !mbar_wait(&s_full[sb], (j >> 1) & 1)) ok = false;
      tc_fence_after();
      if (tr && j == 0) t_data = globaltimer_ns();
      float s[32];
      tmem_ld32(tmem + lane_base + sb * kBC + hh * 32, s);
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      // Scores: bf16(bf16(q.k) * scale); a power-of-two scale needs no second
      // rounding (the product is exact).  The common case (power-of-two scale, no
      // masked key in the half, both warp-uniform) keeps the raw scores: rounding
      // and scaling are monotonic, so the half's max is bf16(max) * scale, and the
      // exponent below takes bf16(s) * (scale * log2e), the same exact product.
      const bool fast = scale_pow2 && all_valid;
      float mxh;
      if (fast) {
        float mx4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int i = 4; i < 32; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], s[i]);
        mxh = bf16_round(fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]))) * p.scale;
      } else {
        float mx4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) mx4[i] = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float v = bf16_round(s[i]) * p.scale;
          if (!scale_pow2) v = bf16_round(v);
          if (!all_valid) v = key_ok(vk, i) ? v : -INFINITY;
          s[i] = v;
          mx4[i & 3] = fmaxf(mx4[i & 3], v);
        }
        mxh = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      }
      s_red[(sb * 2 + hh) * kBR + r] = mxh;
      const bool warp_ok = __all_sync(0xffffffffu, ok);
      if (lane == 0) s_pair_ok[(sb * 2 + hh) * 4 + q] = warp_ok ? 1 : 0;
      // The quarter's two warps (one SM sub-partition): a hardware barrier, cheaper
      // than an mbarrier round trip; the row max of each half is double-buffered
      // by S parity, so neither warp can overwrite a value the other still reads.
      named_bar_sync(4 + q, 64);
      if (s_pair_ok[(sb * 2) * 4 + q] == 0 || s_pair_ok[(sb * 2 + 1) * 4 + q] == 0) {
        ok = false;
        break;
      }
      const float mx = fmaxf(s_red[(sb * 2) * kBR + r], s_red[(sb * 2 + 1) * kBR + r]);
      // Lazy rescale: the exponent base m moves only when the chunk's max exceeds
      // it by more than 8 (P entries stay below e^8 in bf16, whose relative
      // precision does not depend on magnitude); O and l always refer to the same
      // m, so the normalised result is unchanged.  Both halves decide alike.
      const float m_new = fmaxf(m, mx);
      float corr = 1.f;
      if (m == -INFINITY) {
        m = m_new;
      } else if (m_new - m > 8.f) {
        corr = __expf(m - m_new);
        m = m_new;
      }
      const float mb = m == -INFINITY ? 0.f : m * kLog2e;
      float ls4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) ls4[i] = 0.f;
      if (fast) {
        const float c = p.scale * kLog2e;  // exact: scale is a power of two
#pragma unroll
        for (int i = 0; i < 32; i += 2) bf16_round2(s[i], s[i + 1]);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float pv = ex2_approx(fmaf(s[i], c, -mb));  // exp(s - m)
          s[i] = pv;
          ls4[i & 3] += pv;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float pv = ex2_approx(fmaf(s[i], kLog2e, -mb));  // exp(s - m); masked keys give 0
          s[i] = pv;
          ls4[i & 3] += pv;
        }
      }
      l = l * corr + ((ls4[0] + ls4[1]) + (ls4[2] + ls4[3]));
      if (j > 0) {
        // P.V of the previous chunk must be done: P is single-buffered and O may
        // need rescaling.  (A failure is acted on at the next exchange.)
        if (ok && !mbar_wait(p_empty, (j - 1) & 1)) ok = false;
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: rescale when any row of the warp moved
        // (rows whose base did not move multiply by 1).
        if (__any_sync(0xffffffff, corr != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_base + kColO + hh * 128 + c * 32, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(tmem + lane_base + kColO + hh * 128 + c * 32, o);
          }
        }
      }
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {
        uint4 u;
        u.x = pack_bf16x2(s[g4 * 8 + 0], s[g4 * 8 + 1]);
        u.y = pack_bf16x2(s[g4 * 8 + 2], s[g4 * 8 + 3]);
        u.z = pack_bf16x2(s[g4 * 8 + 4], s[g4 * 8 + 5]);
        u.w = pack_bf16x2(s[g4 * 8 + 6], s[g4 * 8 + 7]);
        *reinterpret_cast<uint4*>(sP + p_off(r, hh * 4 + g4)) = u;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (!ok) report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
    // Row sums of the two halves (fixed order: half 0 + half 1).
    s_red[4 * kBR + hh * kBR + r] = l;
    mbar_arrive(&lbar[q]);
    if (ok && !mbar_wait(&lbar[q], 0)) {
      report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
      ok = false;
    }
    const float lt = s_red[4 * kBR + r] + s_red[5 * kBR + r];
    if (ok && nc > 0 && mbar_wait(p_empty, (nc - 1) & 1)) {
      tc_fence_after();
      if (tr) t_loop = globaltimer_ns();
      // Output through shared memory: Q and the K/V ring are free once every MMA
      // is done.  Each warp stages its 32 rows x 128 columns in 128B-swizzled 4 KB
      // slabs (16 KB per warp) and writes them with TMA tensor stores (rows past R
      // are clipped).
      uint8_t* slab0 = smem + (warp - 2) * 4 * 4096;
      if (p.splits == 1) {
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll 1
        for (int jb = 0; jb < 2; ++jb) {
          uint8_t* slab = slab0 + jb * 4096;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            float o[32];
            tmem_ld32(tmem + lane_base + kColO + hh * 128 + jb * 64 + h * 32, o);
#pragma unroll
            for (int g4 = 0; g4 < 4; ++g4) {
              uint4 u;
              u.x = pack_bf16x2(o[g4 * 8 + 0] * inv, o[g4 * 8 + 1] * inv);
              u.y = pack_bf16x2(o[g4 * 8 + 2] * inv, o[g4 * 8 + 3] * inv);
              u.z = pack_bf16x2(o[g4 * 8 + 4] * inv, o[g4 * 8 + 5] * inv);
              u.w = pack_bf16x2(o[g4 * 8 + 6] * inv, o[g4 * 8 + 7] * inv);
              *reinterpret_cast<uint4*>(slab + p_off(lane, h * 4 + g4)) = u;
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int jb = 0; jb < 2; ++jb)
            tma_store_2d(&mp.out, slab0 + jb * 4096, hh * 128 + jb * 64, row0 + q * 32);
          bulk_commit_group();
        }
      } else if (p.cluster_merge) {
        // Two key splits merged here, not by the combine kernel: the row block's two
        // split CTAs form a cluster (rank = split).  Each finishes the O half hh ==
        // rank of its rows.  Once a CTA's MMAs are done its Q, K and P buffers are
        // free, and it tells the peer so; the warps of the other half then push their
        // 32 rows of that half (fp32) and the rows' (m, l) into the peer's K ring and
        // P buffer (one SM-to-SM bulk copy each, completing on the peer's barrier of
        // the lane quarter), and the warps of this CTA's half wait for the peer's
        // rows and merge them with their own O from TMEM in split order with the
        // combine kernel's arithmetic.  No partial goes through global memory.
        const int rank = split;
        const uint32_t peer = (uint32_t)(rank ^ 1);
        if (threadIdx.x == 64) mbar_arrive_cluster(mapa_shared(smem_u32(rfree), peer));
        if (hh != rank) {
          bool sok = true;
          if (lane == 0) sok = mbar_wait_cluster(rfree, 0);
          sok = __shfl_sync(0xffffffffu, sok ? 1 : 0, 0) != 0;
          if (!sok) report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
          uint8_t* stg = sQ + q * kMrgRowBytes;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_base + kColO + hh * 128 + c * 32, o);
#pragma unroll
            for (int g = 0; g < 8; ++g)
              *reinterpret_cast<float4*>(stg + c * 4096 + p_off(lane, g)) =
                  make_float4(o[g * 4], o[g * 4 + 1], o[g * 4 + 2], o[g * 4 + 3]);
          }
          float* mls = reinterpret_cast<float*>(sP + q * kMrgMlBytes);
          mls[2 * lane] = m;
          mls[2 * lane + 1] = lt;
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && sok) {
            const uint32_t pb = mapa_shared(smem_u32(&rrecv[q]), peer);
            bulk_copy_to_peer(mapa_shared(smem_u32(sK + q * kMrgRowBytes), peer), smem_u32(stg), kMrgRowBytes, pb);
            bulk_copy_to_peer(mapa_shared(smem_u32(sP + 4096 + q * kMrgMlBytes), peer), smem_u32(mls), kMrgMlBytes,
                              pb);
          }
        } else {
          // Every lane waits: the phase makes the peer's bulk writes visible to it.
          if (!mbar_wait_cluster(&rrecv[q], 0)) report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
          const uint8_t* rcv = sK + q * kMrgRowBytes;
          const float* mlr = reinterpret_cast<const float*>(sP + 4096 + q * kMrgMlBytes);
          const float mo = mlr[2 * lane], lo = mlr[2 * lane + 1];
          // Split order: split 0's (m, l, O) first.
          const float m0 = split == 0 ? m : mo, l0 = split == 0 ? lt : lo;
          const float m1 = split == 0 ? mo : m, l1 = split == 0 ? lo : lt;
          const float mmax = fmaxf(m0, m1);
          const float w0 = m0 != -INFINITY ? __expf(m0 - mmax) : 0.f;
          const float w1 = m1 != -INFINITY ? __expf(m1 - mmax) : 0.f;
          const float lsum = __fadd_rn(__fmul_rn(l0, w0), __fmul_rn(l1, w1));
          const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
          // bf16 staging, 2 slabs per warp, in the V ring (two slots: the launcher's rule)
          uint8_t* ob = smem + kQBytes + 2 * kKVBytes + (warp - 2) * 8192;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float own[32], oth[32];
            tmem_ld32(tmem + lane_base + kColO + hh * 128 + c * 32, own);
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              const float4 t = *reinterpret_cast<const float4*>(rcv + c * 4096 + p_off(lane, g));
              oth[4 * g] = t.x;
              oth[4 * g + 1] = t.y;
              oth[4 * g + 2] = t.z;
              oth[4 * g + 3] = t.w;
            }
            float o[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float a0 = split == 0 ? own[i] : oth[i], a1 = split == 0 ? oth[i] : own[i];
              o[i] = fmaf(a1, w1, __fmul_rn(a0, w0)) * inv;
            }
            uint8_t* slab = ob + (c >> 1) * 4096;
#pragma unroll
            for (int g4 = 0; g4 < 4; ++g4) {
              uint4 u;
              u.x = pack_bf16x2(o[g4 * 8 + 0], o[g4 * 8 + 1]);
              u.y = pack_bf16x2(o[g4 * 8 + 2], o[g4 * 8 + 3]);
              u.z = pack_bf16x2(o[g4 * 8 + 4], o[g4 * 8 + 5]);
              u.w = pack_bf16x2(o[g4 * 8 + 6], o[g4 * 8 + 7]);
              *reinterpret_cast<uint4*>(slab + p_off(lane, (c & 1) * 4 + g4)) = u;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int jb = 0; jb < 2; ++jb)
              tma_store_2d(&mp.out, ob + jb * 4096, hh * 128 + jb * 64, row0 + q * 32);
            bulk_commit_group();
          }
        }
      } else {
        const int y = split * p.part_rows + row0 + q * 32;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint8_t* slab = slab0 + c * 4096;
          float o[32];
          tmem_ld32(tmem + lane_base + kColO + hh * 128 + c * 32, o);
#pragma unroll
          for (int g = 0; g < 8; ++g)
            *reinterpret_cast<float4*>(slab + p_off(lane, g)) =
                make_float4(o[g * 4], o[g * 4 + 1], o[g * 4 + 2], o[g * 4 + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int c = 0; c < 4; ++c) tma_store_2d(&mp.po, slab0 + c * 4096, hh * 128 + c * 32, y);
          bulk_commit_group();
        }
        // (max, sum) of every row of the padded block; rows past R are padding.
        if (hh == 0) {
          p.part_ml[((size_t)split * p.part_rows + grow) * 2] = m;
          p.part_ml[((size_t)split * p.part_rows + grow) * 2 + 1] = lt;
        }
      }
      // The stores have read the staging slabs before the CTA leaves; their global
      // writes are complete when the grid is, before any dependent grid reads them.
      if (lane == 0) bulk_wait_group_read<0>();
      __syncwarp();
      // Trace record {tag << 32 | cta, entry, grid-dependency wait done, first S
      // ready, last P.V done, output stored, 0, 0} (same layout as attention.cu).
      if (tr) {
        const unsigned long long slot = atomicAdd(p.trace, 1ull);
        if (slot < p.trace[1]) {
          unsigned long long* w = p.trace + 8 + slot * 8;
          w[0] = ((unsigned long long)p.trace_tag << 32) | (blockIdx.y * gridDim.x + blockIdx.x);
          w[1] = t_entry;
          w[2] = t_wait;
          w[3] = t_data;
          w[4] = t_loop;
          w[5] = globaltimer_ns();
          w[6] = 0;
          w[7] = 0;
        }
      }
    } else if (ok && nc > 0) {
      report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
    }
  }

  // Teardown: if the producer stopped early, wait (bounded) for the copies it armed.
  __syncthreads();
  if (s_flag[0] != 0 && warp == 0 && lane == 0) {
    for (int h = 0; h < 2; ++h) {
      const int armed = s_flag[1 + h];
      uint64_t* full = h == 0 ? k_full : v_full;
      for (int st = 0; st < nst && st < armed; ++st) {
        const int uses = (armed - st + nst - 1) / nst;
        if (!mbar_wait(&full[st], (uses - 1) & 1)) report_status(p.status, PI05_DEV_TIMEOUT_DRAIN);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  // Split merge: neither CTA leaves while the other may still signal or copy into
  // its shared memory.
  if (p.cluster_merge) {
    cluster_arrive_release();
    cluster_wait();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool tc_attention_enabled() {
  static int v = [] {
    const char* e = getenv("PI05_ATTN_TC");
    return (e != nullptr && e[0] == '0') ? 0 : 1;
  }();
  return v != 0;
}

int mqa_tc_attention_run(AttnParams p, float* part, size_t part_bytes, int splits, cudaStream_t stream,
                         int (*combine)(const AttnParams&, cudaStream_t)) {
  const int row_blocks = (p.rows + kBR - 1) / kBR;
  const int n_chunks = (p.kv_len + kBC - 1) / kBC;
  int sms = 148;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  if (splits <= 0) {
    // Fill about one wave; fewer splits keep the partial round trip small.
    // PI05_ATTN_TC_SPLITS overrides (tuning).
    static const int force = [] {
      const char* e = getenv("PI05_ATTN_TC_SPLITS");
      return e != nullptr ? atoi(e) : 0;
    }();
    splits = std::max(1, std::min(n_chunks, sms / std::max(1, row_blocks)));
    splits = std::min(splits, 16);
    if (force > 0) splits = force;
  }
  splits = std::min(splits, n_chunks);
  splits = std::min(splits, 32);
  splits = std::max(splits, (n_chunks + kMaxChunks - 1) / kMaxChunks);  // staged mask bytes per CTA
  if ((n_chunks + splits - 1) / splits > kMaxChunks) {
    set_last_error("attention: %d keys exceed %d per split", p.kv_len, kMaxChunks * kBC);
    return PI05_ERR_SHAPE;
  }
  p.splits = splits;
  p.nbuf = (n_chunks + splits - 1) / splits > 1 ? 2 : 1;
  p.part_rows = row_blocks * kBR;  // partial rows padded to whole row blocks
  if (splits > 1) {
    const size_t rows_all = (size_t)splits * p.part_rows;
    const size_t need = rows_all * kD * sizeof(float) + rows_all * 2 * sizeof(float);
    if (part == nullptr || need > part_bytes || (reinterpret_cast<uintptr_t>(part) & 15) != 0) {
      set_last_error("attention: workspace too small (%zu needed)", need);
      return PI05_ERR_WORKSPACE;
    }
    p.part_o = part;
    p.part_ml = part + rows_all * kD;
  }
  TcMaps mp;
  std::memset(&mp, 0, sizeof(mp));
  int rc = make_tmap_bf16_2d(&mp.q, p.q, p.rows, kD, p.q_stride, kBR, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&mp.k, p.k, p.kv_len, kD, p.kv_stride, kBC, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&mp.v, p.v, p.kv_len, kD, p.kv_stride, kBC, 64, true);
  // Two splits merge inside the kernel on 2-CTA clusters; more go through the
  // combine kernel.  (The merge receives into the K ring and stages its bf16 rows in
  // the V ring, so it needs two slots of each.)
  const bool merge = splits == 2 && p.nbuf == 2;
  p.cluster_merge = merge ? 1 : 0;
  if (!rc && (splits == 1 || merge))
    rc = make_tmap_bf16_2d(&mp.out, p.out, p.rows, kD, p.out_stride, 32, 64, true);
  if (!rc && splits > 1) rc = make_tmap_f32_2d(&mp.po, p.part_o, (uint64_t)splits * p.part_rows, kD, kD, 32, 32, true);
  if (rc) return rc;
  const size_t smem = tc_smem_bytes(p.nbuf);
  static bool attr_done[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_done[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(mqa_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tc_smem_bytes(2));
    if (e != cudaSuccess) {
      set_last_error("attention smem attr: %s", cudaGetErrorString(e));
      return PI05_ERR_LAUNCH;
    }
    attr_done[dev] = true;
  }
  if (merge)
    rc = launch_pdl_cluster(mqa_tc_kernel, dim3(row_blocks, splits), dim3(kThreads), smem, stream, pdl_enabled(),
                            dim3(1, 2, 1), mp, p);
  else
    rc = launch_pdl(mqa_tc_kernel, dim3(row_blocks, splits), dim3(kThreads), smem, stream, pdl_enabled(), mp, p);
  if (rc || splits == 1 || merge) return rc;
  return combine(p, stream);
}

}  // namespace pi05
