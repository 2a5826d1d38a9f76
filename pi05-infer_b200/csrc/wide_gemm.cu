// Persistent tcgen05 GEMM for the many-token projections (prefix LM: 968 tokens,
// SigLIP: 256 patches per view, batched denoise at M > 128).
//
//   Y[t, n] = sum_k X[t, k] * W[n, k]
//
// Tokens fill the UMMA M dimension (128 rows per tile) and BN weight rows the N
// dimension (BN = 128, 192 or 256), so TMEM lane r holds token r's BN outputs.
//
// One CTA per SM loops over output tiles (m fastest, so the CTAs resident at a
// time share weight tiles in L2):
//   warp 0      TMA producer: X box 128x64 + two W boxes (BN/2)x64 per k-block
//               into a STAGES-deep ring (128-byte swizzle);
//   warp 1      TMEM owner + MMA issuer: 4 x tcgen05.mma (128 x BN x 16) per
//               k-block into one of two TMEM accumulators (2 x BN columns);
//   warps 2..5  epilogue on the accumulator the MMA warp has finished, while it
//               fills the other one.
//
// Epilogue: each epilogue warp owns 32 token rows (its TMEM lane quarter) and
// works in 64-column slabs (32 rows x 128 B).  A thread reads its row from TMEM,
// applies the fused epilogue and writes the bf16 result into a 128B-swizzled
// slab in shared memory; one lane then stores the slab with a TMA tensor store.
// Row-wise operands (the residual, the RoPE cos/sin rows) arrive the same way,
// by TMA loads into the slab, the first one issued while the mainloop still
// runs.  Every global access of the epilogue is therefore a whole 32x64 box
// instead of 16-byte pieces of 32 different rows, and rows past the token
// count are clipped by the tensor maps.
//
// The two W boxes of a tile are what lets one tile carry the rows an epilogue
// combines (the same pairing as the small-token kernel):
//   GEGLU     : 128 rows of W_gate + the same 128 rows of W_up (BN = 256)
//   QKV_ROPE  : one 256-dim head; columns d and d + 128 are RoPE pairs
//   STORE / GATED_RESID : BN consecutive rows.
//
// Reference ops replaced: the prefix-LM projections of
// pi05_infer/gemma/modeling_gemma.py (GemmaAttention / GemmaMLP forward, :231-249,
// :455-456, :138-148) with the fused QKV+RoPE of prefix_qkv_fused.py:220-246, and
// the SigLIP encoder projections (pi05_infer/siglip/modeling_siglip.py: patch
// embedding, attention in/out projections, MLP fc1/fc2).
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "gemm_epilogue.cuh"
#include "host_util.h"
#include "ptx.cuh"
#include "skinny_gemm.h"
#include "wide_gemm.h"

namespace pi05 {

namespace {

using namespace gemm;
// Epilogue warps EW: 4 (one per TMEM lane quarter), or 8 (two per quarter, each
// taking every other 64-column slab) for STORE / GATED_RESID grids whose tiles
// have a short mainloop, where the epilogue of a single wave is exposed; the 8
// warps' slabs cost one pipeline stage.
template <int EW>
constexpr int wide_threads() {
  return 64 + 32 * EW;
}
constexpr int kWBM = 128;         // tokens per tile
constexpr int kSlabBytes = 4096;  // 32 rows x 64 bf16, 128B swizzle

// Epilogue slabs per warp: QKV keeps cos/sin lo/hi of one 64-column chunk
// (4 slabs); the others double-buffer one slab.
template <int EPI>
constexpr int epi_slabs() {
  return EPI == SK_EPI_QKV_ROPE ? 4 : 2;
}

// B rows a CTA holds per stage: all BN, or half of them when a CTA pair shares
// the tile (cta_group::2).
template <int BN, bool PAIR>
constexpr int wide_b_bytes() {
  return (PAIR ? BN / 2 : BN) * 128;
}

template <int EPI, int BN, int STAGES, int EW, bool PAIR>
constexpr int wide_smem_base() {
  // + 512: barriers, stamps and flags (up to ~300 bytes with 8 epilogue warps).
  return 1024 + STAGES * (kABytes + wide_b_bytes<BN, PAIR>()) + EW * epi_slabs<EPI>() * kSlabBytes + BN * 4 + 512;
}

// Single-CTA STORE tiles also stage the folded LayerNorm's column sums per tile
// when they fit; elsewhere the epilogue reads them from global memory.
template <int EPI, int BN, int STAGES, int EW, bool PAIR>
constexpr bool wide_scol() {
  return !PAIR && EPI == SK_EPI_STORE && wide_smem_base<EPI, BN, STAGES, EW, PAIR>() + BN * 4 <= 232448;
}

template <int EPI, int BN, int STAGES, int EW, bool PAIR>
constexpr int wide_smem_bytes() {
  return wide_smem_base<EPI, BN, STAGES, EW, PAIR>() + (wide_scol<EPI, BN, STAGES, EW, PAIR>() ? BN * 4 : 0);
}

struct WideSched {
  int m_tiles;
  int n_tiles;
  int kb_total;
  int splits;   // split-K (STORE / GATED_RESID only)
};

// A unit's work item: tile (m, n), k-block range [kb0, kb1), and the segment s of
// nseg that cut the tile's K range (split-K; nseg = 1 for a whole tile).
struct WideTile {
  int m, s, n, kb0, kb1, nseg;
};

// Item i of unit `unit` (false past its last).  Tiles are ordered m fastest, so
// units running together share weight tiles.
__device__ __forceinline__ bool wide_item(int unit, int i, int n_units, const WideSched& ws, WideTile& w) {
  const int tiles = ws.m_tiles * ws.n_tiles;
  const int t = unit + i * n_units;
  if (t >= tiles * ws.splits) return false;
  w.m = t % ws.m_tiles;
  const int r = t / ws.m_tiles;
  w.s = r % ws.splits;
  w.n = r / ws.splits;
  w.kb0 = (w.s * ws.kb_total) / ws.splits;
  w.kb1 = ((w.s + 1) * ws.kb_total) / ws.splits;
  w.nseg = ws.splits;
  return true;
}

// Cluster split-K (CSPLIT): the two CTAs of a 2-CTA cluster take K halves of the
// cluster's tile; CTA `rank` takes half `rank`.  One tile per cluster.
__device__ __forceinline__ bool wide_item_cs(int unit, int i, int n_units, const WideSched& ws, int rank,
                                             WideTile& w) {
  const int t = unit + i * n_units;
  if (t >= ws.m_tiles * ws.n_tiles) return false;
  w.m = t % ws.m_tiles;
  w.n = t / ws.m_tiles;
  w.s = rank;
  w.kb0 = (rank * ws.kb_total) / 2;
  w.kb1 = ((rank + 1) * ws.kb_total) / 2;
  w.nseg = 2;
  return true;
}

// Receive buffers of the cluster split-K: per TMEM lane quarter, the peer's fp32
// partial of the 64-column slab this CTA finishes ([32 rows][64], 16-byte chunks
// XOR-swizzled by row so a thread's row reads hit distinct banks).
constexpr int kCsRecvBytes = 4 * 32 * 64 * 4;
__device__ __forceinline__ int cs_off(int r, int c4) { return r * 64 + ((c4 ^ (r & 15)) << 2); }

// Tensor maps of one launch.  out: STORE / GATED_RESID / GEGLU output, or q_out
// for QKV_ROPE.  in0 / in1: residual (GATED_RESID) or cos / sin (QKV_ROPE).
// kc / vc: the K and V cache rows [0, krow0 + m_tok) (QKV_ROPE).  All epilogue
// maps use 32 x 64 boxes with the 128-byte swizzle.
struct WideMaps {
  CUtensorMap x, w0, w1;
  CUtensorMap out, in0, in1, kc, vc;
};

// First weight row of each of the tile's two (BN/2)-row boxes.
template <int EPI, int BN>
__device__ __forceinline__ void wide_rows(int n_tile, int& row0, int& row1) {
  if (EPI == SK_EPI_GEGLU) {
    row0 = n_tile * (BN / 2);
    row1 = row0;
  } else {
    row0 = n_tile * BN;
    row1 = row0 + BN / 2;
  }
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Byte offset of 16-byte chunk g (8 bf16 columns) of row r in a 128B-swizzled slab.
__device__ __forceinline__ uint32_t slab_off(int r, int g) { return (uint32_t)(r * 128 + ((g ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint4 lds16(const uint8_t* slab, int r, int g) {
  return *reinterpret_cast<const uint4*>(slab + slab_off(r, g));
}

__device__ __forceinline__ void sts16(uint8_t* slab, int r, int g, uint4 v) {
  *reinterpret_cast<uint4*>(slab + slab_off(r, g)) = v;
}

// One warp's epilogue state: its 32-row quarter, slabs, slab barriers and the
// phase of each slab barrier (warp-uniform).
struct EpiWarp {
  int q;          // TMEM lane quarter: rows q*32 .. q*32+31 of the tile
  int half;       // which of the quarter's warps (8 epilogue warps): slabs j = half, half + 2, ...
  int step;       // slab stride: 1 with 4 epilogue warps, 2 with 8
  int lane;
  uint8_t* slab;  // epi_slabs<EPI>() consecutive slabs
  uint64_t* bar;  // one barrier per double-buffered slab (QKV uses [0] only)
  uint32_t phase; // bit i: parity of the next completion of bar[i]
};

__device__ __forceinline__ uint8_t* slab_at(const EpiWarp& e, int i) { return e.slab + i * kSlabBytes; }

// Issue (lane 0) the loads of the row operands the tile needs before its
// accumulator is read: residual slab 0, or RoPE cos/sin lo/hi of chunk 0.
template <int EPI, int BN>
__device__ __forceinline__ void wide_epi_prefetch(const SkinnyParams& p, const WideMaps& mp, EpiWarp& e, int n_tile,
                                                  int m0) {
  if (e.lane != 0) return;
  if (EPI == SK_EPI_GATED_RESID) {
    bulk_wait_group_read<0>();
    mbar_arrive_expect_tx(&e.bar[0], kSlabBytes);
    tma_load_2d(slab_at(e, 0), &mp.in0, &e.bar[0], n_tile * BN + e.half * 64, m0 + e.q * 32,
                l2_policy_evict_normal());
  } else if (EPI == SK_EPI_QKV_ROPE) {
    if (n_tile < p.n_q_heads + p.n_kv_heads) {
      const uint64_t pol = l2_policy_evict_last();
      bulk_wait_group_read<0>();
      mbar_arrive_expect_tx(&e.bar[0], 4 * kSlabBytes);
      const int y = m0 + e.q * 32;
      tma_load_2d(slab_at(e, 0), &mp.in0, &e.bar[0], 0, y, pol);
      tma_load_2d(slab_at(e, 1), &mp.in1, &e.bar[0], 0, y, pol);
      tma_load_2d(slab_at(e, 2), &mp.in0, &e.bar[0], 128, y, pol);
      tma_load_2d(slab_at(e, 3), &mp.in1, &e.bar[0], 128, y, pol);
    }
  }
}

__device__ __forceinline__ bool slab_wait(EpiWarp& e, int i, int* status) {
  const bool ok = mbar_wait(&e.bar[i], (e.phase >> i) & 1u);
  e.phase ^= 1u << i;
  if (!ok) report_status(status, PI05_DEV_TIMEOUT_EPILOGUE);
  return ok;
}

// Finish the slab: make the smem writes visible to TMA, store it, commit.
__device__ __forceinline__ void slab_store(const EpiWarp& e, const CUtensorMap* tm, const uint8_t* slab, int x,
                                           int y) {
  fence_proxy_async_smem();
  __syncwarp();
  if (e.lane == 0) {
    tma_store_2d(tm, slab, x, y);
    bulk_commit_group();
  }
}

// STORE / GATED_RESID epilogue features of a launch, fixed per launch (bit mask).
// Each combination the pipelines use is compiled as its own body, so that a
// feature a launch does not have costs no instruction per element: the epilogue
// of a one-tile-per-CTA launch is not overlapped with any mainloop, and the
// per-element work of 4 or 8 epilogue warps over a 128 x BN tile is on its
// critical path.  kEpAny decides every feature at run time (other combinations).
enum : int {
  kEpBias = 1,   // + bias[n] (staged per tile)
  kEpLn = 2,     // folded LayerNorm: rstd * acc - rstd * mean * colsum[n]   (STORE)
  kEpGelu = 4,   // GELU-tanh of the bf16-rounded value                      (STORE)
  kEpPos = 8,    // + pos[token % pos_rows, n]                               (STORE)
  kEpGate = 16,  // residual + y * bf16(gate[n])                             (GATED_RESID)
  kEpSsq = 32,   // row sums of squares of the stored values per 64-column slab
  kEpSum = 64,   // ... and row sums (with kEpSsq)
  kEpAny = 128,
};

template <int EPI>
__device__ __forceinline__ int wide_epi_mask(const SkinnyParams& p) {
  int m = 0;
  if (p.bias != nullptr) m |= kEpBias;
  if (EPI == SK_EPI_STORE && p.ln_colsum != nullptr) m |= kEpLn;
  if (EPI == SK_EPI_STORE && p.act == 1) m |= kEpGelu;
  if (EPI == SK_EPI_STORE && p.pos != nullptr) m |= kEpPos;
  if (EPI == SK_EPI_GATED_RESID && p.gate != nullptr) m |= kEpGate;
  if (p.row_ssq != nullptr) m |= kEpSsq | (p.row_sum != nullptr ? kEpSum : 0);
  return m;
}

// STORE / GATED_RESID (same arithmetic as apply_epilogue), features F.
template <int EPI, int BN, int F>
__device__ __forceinline__ bool wide_epi_rows_f(const SkinnyParams& p, const WideMaps& mp, EpiWarp& e, uint32_t taddr,
                                                int n_tile, int m0, const float* sbias, const float* scol, float ln_rs,
                                                float ln_rm, const float* add) {
  constexpr int NS = BN / 64;
  constexpr bool kAny = (F & kEpAny) != 0;
  const int fm = kAny ? wide_epi_mask<EPI>(p) : F;
  const bool f_bias = (fm & kEpBias) != 0;
  const bool f_ln = EPI == SK_EPI_STORE && (fm & kEpLn) != 0;
  const bool f_gelu = EPI == SK_EPI_STORE && (fm & kEpGelu) != 0;
  const bool f_pos = EPI == SK_EPI_STORE && (fm & kEpPos) != 0;
  const bool f_gate = EPI == SK_EPI_GATED_RESID && (fm & kEpGate) != 0;
  const bool f_ssq = (fm & kEpSsq) != 0;
  const bool f_sum = (fm & kEpSum) != 0;
  const int r = e.lane;
  const int tok = m0 + e.q * 32 + r;
  const int n_valid = p.n_valid > 0 ? p.n_valid : 1 << 30;
  bool ok = true;
#pragma unroll 1
  for (int j = e.half, i = 0; j < NS; j += e.step, ++i) {
    const int b = i & 1;
    uint8_t* slab = slab_at(e, b);
    float ss = 0.f, sx = 0.f;  // row statistics: this row's sum of squares and sum over the slab
    if (EPI == SK_EPI_GATED_RESID) {
      if (j + e.step < NS && e.lane == 0) {  // next residual slab into the other buffer
        bulk_wait_group_read<0>();
        mbar_arrive_expect_tx(&e.bar[b ^ 1], kSlabBytes);
        tma_load_2d(slab_at(e, b ^ 1), &mp.in0, &e.bar[b ^ 1], n_tile * BN + (j + e.step) * 64, m0 + e.q * 32,
                    l2_policy_evict_normal());
      }
    } else {
      if (e.lane == 0) bulk_wait_group_read<1>();  // this buffer's previous store has read it
      __syncwarp();
    }
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      float v[32];
      tmem_ld32(taddr + j * 64 + h * 32, v);
      if (add != nullptr) {  // the other K half of the tile (cluster split-K)
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 t = *reinterpret_cast<const float4*>(add + cs_off(r, h * 8 + c4));
          v[4 * c4] += t.x;
          v[4 * c4 + 1] += t.y;
          v[4 * c4 + 2] += t.z;
          v[4 * c4 + 3] += t.w;
        }
      }
      if (EPI == SK_EPI_GATED_RESID && h == 0) ok = slab_wait(e, b, p.status) && ok;
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {
        const int g = h * 4 + g4;
        const int c = j * 64 + g * 8;  // column within the tile
        const int n = n_tile * BN + c;
        const bool in = n < n_valid;
        float* a = v + g4 * 8;
        if (f_ln) {
          // Folded LayerNorm: column sums staged per tile (zero past n_valid) or read
          // from global memory.
          float cs[8];
          if (scol != nullptr) {
            load8f(scol + c, cs);
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) cs[q] = n + q < n_valid ? p.ln_colsum[n + q] : 0.f;
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) a[q] = a[q] * ln_rs - ln_rm * cs[q];
        }
        if (f_bias) {
          float bi[8];
          load8f(sbias + c, bi);  // staged per tile, zero past n_valid
#pragma unroll
          for (int q = 0; q < 8; ++q) a[q] += bi[q];
        }
        if (f_pos && in) {
          float ps[8];
          load8f(p.pos + (size_t)(tok % p.pos_rows) * p.ldo + n, ps);
#pragma unroll
          for (int q = 0; q < 8; ++q) a[q] += ps[q];
        }
        if (f_gelu) {
#pragma unroll
          for (int q = 0; q < 8; q += 2) bf16_round2(a[q], a[q + 1]);
#pragma unroll
          for (int q = 0; q < 8; ++q) a[q] = gelu_tanh_fast(a[q]);
        }
        if (EPI == SK_EPI_GATED_RESID) {
          float rs[8];
          unpack8(lds16(slab, r, g), rs);
#pragma unroll
          for (int q = 0; q < 8; q += 2) bf16_round2(a[q], a[q + 1]);
          if (f_gate && in) {
            float gt[8];
            load8f(p.gate + n, gt);
#pragma unroll
            for (int q = 0; q < 8; q += 2) bf16_round2(gt[q], gt[q + 1]);
#pragma unroll
            for (int q = 0; q < 8; ++q) a[q] = rs[q] + a[q] * gt[q];
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) a[q] = rs[q] + a[q];
          }
        }
        const uint4 pk = pack8(a);
        if (f_ssq && in) {  // the stored (bf16) values
          float q8[8];
          unpack8(pk, q8);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            ss = fmaf(q8[q], q8[q], ss);
            if (f_sum) sx += q8[q];
          }
        }
        sts16(slab, r, g, pk);
      }
    }
    if (f_ssq && tok < p.m_tok && n_tile * BN + j * 64 < n_valid) {
      p.row_ssq[(size_t)(n_tile * (BN / 64) + j) * p.ssq_ld + tok] = ss;
      if (f_sum) p.row_sum[(size_t)(n_tile * (BN / 64) + j) * p.ssq_ld + tok] = sx;
    }
    slab_store(e, &mp.out, slab, n_tile * BN + j * 64, m0 + e.q * 32);
  }
  return ok;
}

// The body for the launch's feature mask (the combinations the SigLIP encoder, the
// prefix LM and the plain linear ops use; kEpAny otherwise).
template <int EPI, int BN>
__device__ __forceinline__ bool wide_epi_rows(const SkinnyParams& p, const WideMaps& mp, EpiWarp& e, uint32_t taddr,
                                              int n_tile, int m0, const float* sbias, const float* scol, float ln_rs,
                                              float ln_rm, const float* add = nullptr) {
#define PI05_WIDE_EPI(F) wide_epi_rows_f<EPI, BN, (F)>(p, mp, e, taddr, n_tile, m0, sbias, scol, ln_rs, ln_rm, add)
  const int m = wide_epi_mask<EPI>(p);
  if (EPI == SK_EPI_STORE) {
    switch (m) {
      case 0: return PI05_WIDE_EPI(0);
      case kEpBias: return PI05_WIDE_EPI(kEpBias);
      case kEpBias | kEpLn: return PI05_WIDE_EPI(kEpBias | kEpLn);
      case kEpBias | kEpLn | kEpGelu: return PI05_WIDE_EPI(kEpBias | kEpLn | kEpGelu);
      case kEpBias | kEpGelu: return PI05_WIDE_EPI(kEpBias | kEpGelu);
      case kEpBias | kEpPos | kEpSsq | kEpSum: return PI05_WIDE_EPI(kEpBias | kEpPos | kEpSsq | kEpSum);
      default: return PI05_WIDE_EPI(kEpAny);
    }
  }
  switch (m) {
    case 0: return PI05_WIDE_EPI(0);
    case kEpGate: return PI05_WIDE_EPI(kEpGate);
    case kEpSsq: return PI05_WIDE_EPI(kEpSsq);
    case kEpBias: return PI05_WIDE_EPI(kEpBias);
    case kEpBias | kEpSsq | kEpSum: return PI05_WIDE_EPI(kEpBias | kEpSsq | kEpSum);
    default: return PI05_WIDE_EPI(kEpAny);
  }
#undef PI05_WIDE_EPI
}

// GEGLU: TMEM columns [0, 128) are gate rows, [128, 256) the matching up rows.
__device__ __forceinline__ void wide_epi_geglu(const WideMaps& mp, EpiWarp& e, uint32_t taddr, int n_tile, int m0,
                                               float rs) {
  const int r = e.lane;
#pragma unroll 1
  for (int j = 0; j < 2; ++j) {
    uint8_t* slab = slab_at(e, j);
    if (e.lane == 0) bulk_wait_group_read<1>();
    __syncwarp();
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      float g[32], u[32];
      tmem_ld32(taddr + j * 64 + h * 32, g);
      tmem_ld32(taddr + 128 + j * 64 + h * 32, u);
#pragma unroll
      for (int i = 0; i < 32; ++i) {  // folded norm: the row's rstd (1 otherwise)
        g[i] *= rs;
        u[i] *= rs;
      }
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {
        float o[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) o[jj] = gelu_tanh_f(bf16_round(g[g4 * 8 + jj])) * u[g4 * 8 + jj];
        sts16(slab, r, h * 4 + g4, pack8(o));
      }
    }
    slab_store(e, &mp.out, slab, n_tile * 128 + j * 64, m0 + e.q * 32);
  }
}

// QKV_ROPE, one 256-dim head per tile (n_kv_heads == 1): q / k heads are rotated
// (pairs d, d + 128) into q_out / the K cache; the v head is copied to the V cache.
__device__ __forceinline__ bool wide_epi_qkv(const SkinnyParams& p, const WideMaps& mp, EpiWarp& e, uint32_t taddr,
                                             int head, int m0, float rs) {
  const int r = e.lane;
  const int y_q = m0 + e.q * 32;
  const int y_kv = p.krow0 + m0 + e.q * 32;
  bool ok = true;
  if (head < p.n_q_heads + p.n_kv_heads) {
    const bool is_q = head < p.n_q_heads;
    const CUtensorMap* dst = is_q ? &mp.out : &mp.kc;
    const int x0 = is_q ? head * 256 : 0;
    const int y = is_q ? y_q : y_kv;
    uint8_t* s_cl = slab_at(e, 0);
    uint8_t* s_sl = slab_at(e, 1);
    uint8_t* s_ch = slab_at(e, 2);
    uint8_t* s_sh = slab_at(e, 3);
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      if (c == 1 && e.lane == 0) {  // chunk 1's cos/sin once chunk 0's stores have read the slabs
        const uint64_t pol = l2_policy_evict_last();
        bulk_wait_group_read<0>();
        mbar_arrive_expect_tx(&e.bar[0], 4 * kSlabBytes);
        tma_load_2d(s_cl, &mp.in0, &e.bar[0], 64, y_q, pol);
        tma_load_2d(s_sl, &mp.in1, &e.bar[0], 64, y_q, pol);
        tma_load_2d(s_ch, &mp.in0, &e.bar[0], 192, y_q, pol);
        tma_load_2d(s_sh, &mp.in1, &e.bar[0], 192, y_q, pol);
      }
      ok = slab_wait(e, 0, p.status) && ok;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float lo[32], hi[32];
        tmem_ld32(taddr + c * 64 + h * 32, lo);
        tmem_ld32(taddr + 128 + c * 64 + h * 32, hi);
#pragma unroll
        for (int i = 0; i < 32; ++i) {  // folded norm: the row's rstd (1 otherwise)
          lo[i] *= rs;
          hi[i] *= rs;
        }
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          const int g = h * 4 + g4;
          float cl[8], sl[8], ch[8], sh[8], olo[8], ohi[8];
          unpack8(lds16(s_cl, r, g), cl);
          unpack8(lds16(s_sl, r, g), sl);
          unpack8(lds16(s_ch, r, g), ch);
          unpack8(lds16(s_sh, r, g), sh);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const float xl = bf16_round(lo[g4 * 8 + jj]), xh = bf16_round(hi[g4 * 8 + jj]);
            olo[jj] = xl * cl[jj] - xh * sl[jj];
            ohi[jj] = xh * ch[jj] + xl * sh[jj];
          }
          // Each thread overwrites only its own row's chunks, which it has just read.
          sts16(s_cl, r, g, pack8(olo));
          sts16(s_ch, r, g, pack8(ohi));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (e.lane == 0) {
        tma_store_2d(dst, s_cl, x0 + c * 64, y);
        tma_store_2d(dst, s_ch, x0 + 128 + c * 64, y);
        bulk_commit_group();
      }
    }
  } else {
    if (e.lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      uint8_t* slab = slab_at(e, j & 1);
      if (j > 1) {
        if (e.lane == 0) bulk_wait_group_read<1>();
        __syncwarp();
      }
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float v[32];
        tmem_ld32(taddr + j * 64 + h * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= rs;
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) sts16(slab, r, h * 4 + g4, pack8(v + g4 * 8));
      }
      slab_store(e, &mp.vc, slab, j * 64, y_kv);
    }
  }
  return ok;
}

// PAIR: the two CTAs of a 2-CTA cluster share each tile of 256 tokens x BN (= 256)
// columns.  CTA r loads tokens r*128 .. r*128+127 of the tile and weight box r
// (w0 rows for r = 0, w1 rows for r = 1); the even CTA (leader) issues
// tcgen05.mma.cta_group::2 with M = 256, which reads both CTAs' shared memory and
// accumulates into both CTAs' TMEM (CTA r: rows r*128 ..), so each SM streams
// 32 KB of operands per k-block instead of 48 KB for the same FLOPs.  Both CTAs'
// TMA loads (cta_group::2 form, one destination each) complete on the leader's full
// barrier, which the leader arms for both; the leader's commits arrive on both
// CTAs' barriers (one commit with a two-CTA mask); the epilogues are per CTA, the odd CTA's
// warps signalling "accumulator drained" to the leader remotely.
template <int EPI, int BN, int STAGES, int EW, bool PAIR, bool CSPLIT = false>
__global__ void __launch_bounds__(wide_threads<EW>(), 1)
    wide_gemm_kernel(const __grid_constant__ WideMaps mp, const SkinnyParams p, const WideSched ws) {
  constexpr int kBBytes = wide_b_bytes<BN, PAIR>();
  constexpr int kStageBytes = kABytes + kBBytes;
  constexpr uint32_t kTmemCols = BN == 192 ? 512 : 2 * BN;  // a power of two
  constexpr uint32_t kIdesc = umma_idesc_bf16(PAIR ? 2 * kWBM : kWBM, BN);
  static_assert(!PAIR || BN == 256, "CTA pairs use 256-wide tiles");
  constexpr int kSlabs = epi_slabs<EPI>();
  constexpr int kEW = EW;
  static_assert(EW == 4 || ((EPI == SK_EPI_STORE || EPI == SK_EPI_GATED_RESID) && EW == 8), "epilogue warps");
  constexpr int kET = kEW * 32;  // epilogue threads
  static_assert(BN == 128 || BN == 192 || BN == 256, "tile width");
  static_assert(!CSPLIT || (!PAIR && BN == 128 && EW == 8 && (EPI == SK_EPI_STORE || EPI == SK_EPI_GATED_RESID)),
                "cluster split-K: one 64-column slab per epilogue warp");
  static_assert((EPI != SK_EPI_GEGLU && EPI != SK_EPI_QKV_ROPE) || BN == 256, "paired epilogues use BN = 256");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kABytes;
  uint8_t* sEpi = smem + STAGES * kStageBytes;  // kEW warps x kSlabs slabs, 1024-aligned
  uint8_t* sRecv = sEpi + kEW * kSlabs * kSlabBytes;  // CSPLIT: kCsRecvBytes of peer partials
  float* sbias = reinterpret_cast<float*>(sRecv + (CSPLIT ? kCsRecvBytes : 0));  // [BN] this tile's bias
  constexpr bool kScol = wide_scol<EPI, BN, STAGES, EW, PAIR>();
  float* scol = sbias + BN;  // [BN] folded LayerNorm column sums (kScol)
  uint64_t* full = reinterpret_cast<uint64_t*>(sbias + (kScol ? 2 : 1) * BN);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2] accumulator ready (MMA commit)
  uint64_t* acce = accf + 2;        // [2] accumulator drained (128 epilogue arrivals)
  uint64_t* mdone = acce + 2;       // all MMAs of this CTA complete
  uint64_t* sbar = mdone + 1;       // [kEW warps][2] epilogue slab loads
  uint64_t* rbar = sbar + 2 * kEW;  // CSPLIT: [4] peer partial of a lane quarter received
  unsigned long long* s_stamp = reinterpret_cast<unsigned long long*>(rbar + (CSPLIT ? 4 : 0));  // [2] trace
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(s_stamp + 2);
  int* s_flag = reinterpret_cast<int*>(s_tmem + 1);  // [0] abort, [2] k-blocks armed

  const uint64_t t_entry = (p.trace != nullptr) ? globaltimer_ns() : 0;
  uint64_t t_setup = 0, t_acc = 0, t_epi = 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work units: CTAs, or CTA pairs (ws.m_tiles then counts 256-token pair tiles).
  const int rank = (PAIR || CSPLIT) ? (int)cluster_ctarank() : 0;
  const bool leader = rank == 0;
  const int unit0 = (PAIR || CSPLIT) ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int n_units = (PAIR || CSPLIT) ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  auto next_item = [&](int item, WideTile& w) -> bool {
    return CSPLIT ? wide_item_cs(unit0, item, n_units, ws, rank, w) : wide_item(unit0, item, n_units, ws, w);
  };
  const int cta_m_tiles = PAIR ? 2 * ws.m_tiles : ws.m_tiles;  // 128-token tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);  // pairs: the leader's, completed by both CTAs' copies
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], PAIR ? 2 * kEW : kET);  // pairs: one arrival per epilogue warp of either CTA
    }
    mbar_init(mdone, 1);
    for (int i = 0; i < 2 * kEW; ++i) mbar_init(&sbar[i], 1);
    if (CSPLIT) {
      for (int i = 0; i < 4; ++i) {
        mbar_init(&rbar[i], 1);
        mbar_arrive_expect_tx(&rbar[i], 32 * 64 * 4);  // one use per launch: one tile per cluster
      }
    }
    s_flag[0] = 0;
    s_flag[2] = 0;
    s_stamp[0] = 0;
    s_stamp[1] = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&mp.x);
    prefetch_tmap(&mp.w0);
    prefetch_tmap(&mp.w1);
  }
  if (warp == 2 && lane == 0) {
    prefetch_tmap(&mp.out);
    if (EPI == SK_EPI_GATED_RESID || EPI == SK_EPI_QKV_ROPE) prefetch_tmap(&mp.in0);
    if (EPI == SK_EPI_QKV_ROPE) {
      prefetch_tmap(&mp.in1);
      prefetch_tmap(&mp.kc);
      prefetch_tmap(&mp.vc);
    }
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(s_tmem, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(s_tmem, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR || CSPLIT) {
    // Both CTAs' barriers are initialised before either signals the other.
    cluster_arrive_release();
    cluster_wait();
  }
  tc_fence_after();
  const uint32_t tmem = *s_tmem;
  if (p.trace != nullptr) t_setup = globaltimer_ns();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_normal();
      const uint64_t pol_x = l2_policy_evict_last();
      int it = 0;
      bool waited = false;
      // Pairs: every copy completes on the leader's barrier of the stage.
      const uint32_t lead_full = PAIR ? mapa_shared(smem_u32(full), 0) : 0u;
      auto load = [&](void* dst, const CUtensorMap* tm, int st, int x, int y, uint64_t pol) {
        if (PAIR)
          tma_load_2d_pair(dst, tm, lead_full + (uint32_t)st * 8u, x, y, pol);
        else
          tma_load_2d(dst, tm, &full[st], x, y, pol);
      };
      // The leader arms its barrier for both CTAs' bytes; the odd CTA arms none.
      auto arm = [&](int st) {
        if (!PAIR)
          mbar_arrive_expect_tx(&full[st], kStageBytes);
        else if (leader)
          mbar_arrive_expect_tx(&full[st], 2 * kStageBytes);
      };
      // W boxes of a stage: both (one CTA per tile) or this CTA's (pairs).
      auto load_w = [&](int st, int kb, int row0, int row1) {
        if (!PAIR || leader) load(sB + st * kBBytes, &mp.w0, st, kb * kBK, row0, pol_w);
        if (!PAIR || !leader) load(sB + st * kBBytes + (PAIR ? 0 : kBBytes / 2), &mp.w1, st, kb * kBK, row1, pol_w);
      };
      WideTile wt;
      for (int item = 0; next_item(item, wt); ++item) {
        const int m = PAIR ? 2 * wt.m + rank : wt.m;  // this CTA's 128-token tile
        int row0, row1;
        wide_rows<EPI, BN>(wt.n, row0, row1);
        // First tile: weights do not depend on the previous kernel, so the first
        // ring's worth of W boxes is issued before the grid-dependency wait.
        int kb = wt.kb0;
        if (!waited) {
          const int pre = min(STAGES, wt.kb1 - wt.kb0);
          for (int i = 0; i < pre; ++i) {
            arm(i);
            load_w(i, wt.kb0 + i, row0, row1);
          }
          pdl_wait();
          waited = true;
          if (p.trace != nullptr) s_stamp[0] = globaltimer_ns();
          for (int i = 0; i < pre; ++i) load(sA + i * kABytes, &mp.x, i, (wt.kb0 + i) * kBK, m * kWBM, pol_x);
          kb = wt.kb0 + pre;
          it = pre;
        }
        for (; kb < wt.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1)) {
            report_status(p.status, PI05_DEV_TIMEOUT_PRODUCER);
            s_flag[0] = 1;
            break;
          }
          arm(s);
          load_w(s, kb, row0, row1);
          load(sA + s * kABytes, &mp.x, s, kb * kBK, m * kWBM, pol_x);
        }
        if (s_flag[0] != 0) break;
      }
      if (!waited) pdl_wait();
      s_flag[2] = it;
    }
  } else if (warp == 1) {
    if (PAIR && !leader) {
      // Odd CTA of a pair: the leader issues every MMA.
    } else if (lane == 0) {
      int it = 0, lt = 0;
      bool ok = true;
      WideTile wt;
      for (int item = 0; ok && next_item(item, wt); ++item, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait(&acce[buf], ((lt >> 1) & 1) ^ 1)) {
          report_status(p.status, PI05_DEV_TIMEOUT_MMA);
          ok = false;
          break;
        }
        tc_fence_after();
        if (p.trace != nullptr && lt == 0) s_stamp[1] = globaltimer_ns();
        const uint32_t d = tmem + (uint32_t)(buf * BN);
        for (int kb = wt.kb0; kb < wt.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          // Pairs: the odd CTA's copies complete the phase too.
          if (!(PAIR ? mbar_wait_cluster(&full[s], (it / STAGES) & 1) : mbar_wait(&full[s], (it / STAGES) & 1))) {
            report_status(p.status, PI05_DEV_TIMEOUT_MMA);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + s * kABytes);
          const uint32_t b0 = smem_u32(sB + s * kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint32_t acc = (kb > wt.kb0 || kk > 0) ? 1u : 0u;
            if (PAIR)
              umma_bf16_pair(d, umma_sdesc_sw128(a0 + kk * 32), umma_sdesc_sw128(b0 + kk * 32), kIdesc, acc);
            else
              umma_bf16(d, umma_sdesc_sw128(a0 + kk * 32), umma_sdesc_sw128(b0 + kk * 32), kIdesc, acc);
          }
          if (PAIR)
            umma_commit_pair(&empty[s], 0x3);
          else
            umma_commit(&empty[s]);
        }
        if (ok) {
          if (PAIR)
            umma_commit_pair(&accf[buf], 0x3);
          else
            umma_commit(&accf[buf]);
        }
      }
      if (!ok) s_flag[0] = 1;
      // Every MMA issued by this thread has completed once mdone fires.
      if (PAIR)
        umma_commit_pair(mdone, 0x3);
      else
        umma_commit(mdone);
      if (!mbar_wait(mdone, 0)) report_status(p.status, PI05_DEV_TIMEOUT_DRAIN);
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter = warp % 4, one token row per thread.
    pdl_wait();
    EpiWarp e;
    e.q = warp & 3;
    e.half = (warp - 2) >> 2;
    e.step = kEW / 4;
    e.lane = lane;
    e.slab = sEpi + (warp - 2) * kSlabs * kSlabBytes;
    e.bar = sbar + (warp - 2) * 2;
    e.phase = 0;
    int lt = 0;
    WideTile wt;
    for (int item = 0; next_item(item, wt); ++item, ++lt) {
      const int m = PAIR ? 2 * wt.m + rank : wt.m, n = wt.n;  // this CTA's 128-token tile
      const int buf = lt & 1;
      // CSPLIT: a warp whose slab the peer finishes loads no residual.
      if (!CSPLIT || e.half == rank) wide_epi_prefetch<EPI, BN>(p, mp, e, n, m * kWBM);
      if ((EPI == SK_EPI_STORE || EPI == SK_EPI_GATED_RESID) && (p.bias != nullptr || p.ln_colsum != nullptr)) {
        // Stage the tile's bias (and folded LayerNorm column sums) once; the
        // epilogue reads them as shared-memory broadcasts.
        const int et = threadIdx.x - 64;
        named_bar_sync(1, kET);  // the previous tile's epilogue is done with sbias / scol
        for (int i = et; i < BN; i += kET) {
          const int col = n * BN + i;
          if (p.bias != nullptr) sbias[i] = col < p.n_valid ? p.bias[col] : 0.f;
          if (kScol && p.ln_colsum != nullptr) scol[i] = col < p.n_valid ? p.ln_colsum[col] : 0.f;
        }
        named_bar_sync(1, kET);
      }
      // Folded norm (q|k|v, gate/up): rstd of this thread's token row from the
      // producer's per-slab sums of squares, loaded while the mainloop runs.
      float rs = 1.f;
      if ((EPI == SK_EPI_GEGLU || EPI == SK_EPI_QKV_ROPE) && p.fold_ssq != nullptr) {
        const int tok = m * kWBM + e.q * 32 + lane;
        float ss = 0.f;
        if (tok < p.m_tok) {
#pragma unroll 8
          for (int j = 0; j < p.fold_parts; ++j) ss += __ldcg(p.fold_ssq + (size_t)j * p.fold_ld + tok);
        }
        rs = tok < p.m_tok ? rsqrtf(ss / (float)p.fold_d + p.fold_eps) : 0.f;
      }
      // Folded LayerNorm (STORE): rstd and rstd * mean of the row from the producer's
      // per-slab sums and sums of squares.
      float ln_rs = 1.f, ln_rm = 0.f;
      if (EPI == SK_EPI_STORE && p.ln_sum != nullptr) {
        const int tok = m * kWBM + e.q * 32 + lane;
        float s1 = 0.f, s2 = 0.f;
        if (tok < p.m_tok) {
#pragma unroll 6
          for (int j = 0; j < p.fold_parts; ++j) {
            s1 += __ldcg(p.ln_sum + (size_t)j * p.fold_ld + tok);
            s2 += __ldcg(p.fold_ssq + (size_t)j * p.fold_ld + tok);
          }
        }
        const float mean = s1 / (float)p.fold_d;
        const float var = fmaxf(s2 / (float)p.fold_d - mean * mean, 0.f);
        ln_rs = tok < p.m_tok ? rsqrtf(var + p.fold_eps) : 0.f;
        ln_rm = ln_rs * mean;
      }
      if (!mbar_wait(&accf[buf], (lt >> 1) & 1)) {
        report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
        break;
      }
      tc_fence_after();
      if (p.trace != nullptr && lt == 0) t_acc = globaltimer_ns();
      const uint32_t taddr = tmem + ((uint32_t)(e.q * 32) << 16) + (uint32_t)(buf * BN);
      bool ok = true;
      if (EPI == SK_EPI_GEGLU)
        wide_epi_geglu(mp, e, taddr, n, m * kWBM, rs);
      else if (EPI == SK_EPI_QKV_ROPE)
        ok = wide_epi_qkv(p, mp, e, taddr, n, m * kWBM, rs);
      else {
        bool finish = true;
        const float* add = nullptr;
        if (CSPLIT) {
          // The tile's two K halves: this CTA finishes slab `rank` (64 columns), the
          // peer slab rank ^ 1.  A warp of the other slab sends its 32 rows of it,
          // fp32, straight into the peer's receive buffer of its lane quarter (one
          // 8 KB SM-to-SM copy completing on the peer's barrier); a warp of this
          // CTA's slab waits for the peer's rows and adds them to its accumulator.
          // a + b == b + a, so both CTAs' sums are the same whichever sent which.
          const int peer = rank ^ 1;
          if (e.half != rank) {
            uint8_t* stg = slab_at(e, 0);  // the warp's two slabs: 8 KB
            float* stgf = reinterpret_cast<float*>(stg);
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
              float v[32];
              tmem_ld32(taddr + e.half * 64 + h * 32, v);
#pragma unroll
              for (int c4 = 0; c4 < 8; ++c4)
                *reinterpret_cast<float4*>(stgf + cs_off(lane, h * 8 + c4)) =
                    make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0)
              bulk_copy_to_peer(mapa_shared(smem_u32(sRecv) + (uint32_t)(e.q * 8192), (uint32_t)peer), smem_u32(stg),
                                8192u, mapa_shared(smem_u32(&rbar[e.q]), (uint32_t)peer));
            finish = false;
          } else {
            if (!mbar_wait_cluster(&rbar[e.q], 0)) {
              report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
              ok = false;
            }
            add = reinterpret_cast<const float*>(sRecv + e.q * 8192);
          }
        } else if (wt.nseg > 1) {
          // Publish this segment's partial, take a ticket; the segment taking the
          // last ticket sums every segment's partial in segment order into its
          // TMEM accumulator and runs the epilogue.  No CTA waits for another.
          // Partials move warp-cooperatively through slab 1 (slab 0 may hold the
          // prefetched residual): a thread owns a TMEM row, while 8 lanes together
          // move one 128-byte line of a row in global memory.
          const int tile_mn = n * cta_m_tiles + m;
          float* part = p.accum + (size_t)tile_mn * ws.splits * kWBM * BN;
          uint8_t* xs = slab_at(e, 1);
          const int g = lane & 7;  // this lane's 16-byte piece of a 128-byte line
          if (e.lane == 0) bulk_wait_group_read<0>();  // slab 1's last TMA store has read it
          __syncwarp();
          const size_t my_rows = (size_t)wt.s * kWBM + e.q * 32;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            if (((c >> 1) % e.step) != e.half) continue;  // the quarter's other warp takes this slab
            float v[32];
            tmem_ld32(taddr + c * 32, v);
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4)
              *reinterpret_cast<float4*>(xs + lane * 128 + ((q4 ^ (lane & 7)) << 4)) =
                  make_float4(v[4 * q4], v[4 * q4 + 1], v[4 * q4 + 2], v[4 * q4 + 3]);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int rr = (lane >> 3) + 4 * i;
              __stcg(reinterpret_cast<float4*>(part + (my_rows + rr) * BN + c * 32 + g * 4),
                     *reinterpret_cast<const float4*>(xs + rr * 128 + ((g ^ (rr & 7)) << 4)));
            }
            __syncwarp();
          }
          __threadfence();
          named_bar_sync(1, kET);
          if (threadIdx.x == 64) {
            const int old = atomicAdd(p.counters + tile_mn, 1);
            const int last = old == wt.nseg - 1 ? 1 : 0;
            if (last) atomicExch(p.counters + tile_mn, 0);  // re-armed for the next launch
            s_flag[1] = last;
          }
          named_bar_sync(1, kET);
          finish = s_flag[1] != 0;
          named_bar_sync(1, kET);  // s_flag[1] is rewritten by the next split tile
          if (finish) {
            __threadfence();
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
              if (((c >> 1) % e.step) != e.half) continue;
              float own[32], acc[32];
              tmem_ld32(taddr + c * 32, own);
#pragma unroll
              for (int i = 0; i < 32; ++i) acc[i] = 0.f;
#pragma unroll 1
              for (int sg = 0; sg < wt.nseg; ++sg) {
                if (sg == wt.s) {
#pragma unroll
                  for (int i = 0; i < 32; ++i) acc[i] += own[i];
                  continue;
                }
                const size_t rows = (size_t)sg * kWBM + e.q * 32;
                float4 t[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const int rr = (lane >> 3) + 4 * i;
                  t[i] = __ldcg(reinterpret_cast<const float4*>(part + (rows + rr) * BN + c * 32 + g * 4));
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                  const int rr = (lane >> 3) + 4 * i;
                  *reinterpret_cast<float4*>(xs + rr * 128 + ((g ^ (rr & 7)) << 4)) = t[i];
                }
                __syncwarp();
#pragma unroll
                for (int q4 = 0; q4 < 8; ++q4) {
                  const float4 u = *reinterpret_cast<const float4*>(xs + lane * 128 + ((q4 ^ (lane & 7)) << 4));
                  acc[4 * q4] += u.x;
                  acc[4 * q4 + 1] += u.y;
                  acc[4 * q4 + 2] += u.z;
                  acc[4 * q4 + 3] += u.w;
                }
                __syncwarp();
              }
              tmem_st32(taddr + c * 32, acc);
            }
          }
        }
        if (finish) {
          ok = wide_epi_rows<EPI, BN>(p, mp, e, taddr, n, m * kWBM, sbias, kScol ? scol : nullptr, ln_rs, ln_rm,
                                      add) &&
               ok;
        } else if (CSPLIT) {
          // Sender: no residual was prefetched.
        } else if (EPI == SK_EPI_GATED_RESID && e.lane == 0) {
          // The residual slab prefetched for this tile is not consumed: retire its load.
          ok = slab_wait(e, 0, p.status);
        } else if (EPI == SK_EPI_GATED_RESID) {
          e.phase ^= 1u;
        }
      }
      tc_fence_before();
      if (PAIR) {
        // One arrival per warp on the leader's barrier (remote for the odd CTA).
        __syncwarp();
        if (lane == 0) {
          if (leader)
            mbar_arrive(&acce[buf]);
          else
            mbar_arrive_cluster(mapa_shared(smem_u32(&acce[buf]), 0));
        }
      } else {
        mbar_arrive(&acce[buf]);
      }
      if (!ok) break;
    }
    // All of this warp's tensor stores complete (and stop reading shared memory)
    // before the CTA exits.
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
    if (p.trace != nullptr) t_epi = globaltimer_ns();
  }

  // Teardown.  If the producer stopped early, wait (bounded) for the copies it
  // armed before shared memory is released.
  __syncthreads();
  if (s_flag[0] != 0 && warp == 0 && lane == 0 && (!PAIR || leader)) {
    const int armed = s_flag[2];
    for (int s = 0; s < STAGES && s < armed; ++s) {
      const int uses = (armed - s + STAGES - 1) / STAGES;  // armings of stage s
      if (!mbar_wait(&full[s], (uses - 1) & 1)) report_status(p.status, PI05_DEV_TIMEOUT_DRAIN);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (PAIR || CSPLIT) {
    // Neither CTA leaves (releasing shared memory the leader's MMAs read, or the
    // barriers the other signals, or a partial the other still copies out) before
    // both are done; the leader's MMAs have all completed (mdone) before it arrives,
    // and a CSPLIT CTA's epilogue has received the peer's partial.
    cluster_arrive_release();
    cluster_wait();
  }
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem, kTmemCols);
    else
      tmem_dealloc(tmem, kTmemCols);
  }
  // Trace record {tag << 32 | cta, entry, setup done, first X TMA after the grid
  // dependency wait, MMA passed the first accumulator-free wait, first
  // accumulator ready, epilogue done (stores complete), exit}.
  if (p.trace != nullptr && threadIdx.x == 64) {
    const unsigned long long slot = atomicAdd(p.trace, 1ull);
    if (slot < p.trace[1]) {
      unsigned long long* w = p.trace + 8 + slot * 8;
      w[0] = ((unsigned long long)p.trace_tag << 32) | blockIdx.x;
      w[1] = t_entry;
      w[2] = t_setup;
      w[3] = s_stamp[0];
      w[4] = s_stamp[1];
      w[5] = t_acc;
      w[6] = t_epi;
      w[7] = globaltimer_ns();
    }
  }
}

int wide_sms() {
  static int cached[16] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 16) cached[dev] = n;
  return n;
}

template <int EPI, int BN, int STAGES, int EW, bool PAIR = false, bool CSPLIT = false>
int wide_launch(const SkinnyParams& p, const WideSched& ws, const WideMaps& mp, cudaStream_t stream) {
  constexpr int kSmem = wide_smem_bytes<EPI, BN, STAGES, EW, PAIR>() + (CSPLIT ? kCsRecvBytes : 0);
  static_assert(kSmem <= 232448, "shared memory per block");
  auto kern = wide_gemm_kernel<EPI, BN, STAGES, EW, PAIR, CSPLIT>;
  static bool attr_done[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) {
      set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return PI05_ERR_LAUNCH;
    }
    attr_done[dev] = true;
  }
  const int total = ws.m_tiles * ws.n_tiles * ws.splits;
  if (PAIR) {
    // Persistent pairs: as many as can be resident at once (a GPC with an odd
    // number of free SMs leaves one unpaired), or a late wave doubles the time.
    static int max_pairs[16] = {0};
    if (dev < 16 && max_pairs[dev] == 0) {
      cudaLaunchConfig_t cfg;
      std::memset(&cfg, 0, sizeof(cfg));
      cfg.gridDim = dim3(2 * (wide_sms() / 2));
      cfg.blockDim = dim3(wide_threads<EW>());
      cfg.dynamicSmemBytes = kSmem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = wide_sms() / 2;
      }
      max_pairs[dev] = n;
    }
    const int pairs = std::min(total, dev < 16 ? max_pairs[dev] : wide_sms() / 2);
    return launch_pdl_cluster(kern, dim3(2 * pairs), dim3(wide_threads<EW>()), kSmem, stream, pdl_enabled(),
                              dim3(2, 1, 1), mp, p, ws);
  }
  if (CSPLIT)  // one tile per 2-CTA cluster (the launcher checks that they fit one wave)
    return launch_pdl_cluster(kern, dim3(2 * ws.m_tiles * ws.n_tiles), dim3(wide_threads<EW>()), kSmem, stream,
                              pdl_enabled(), dim3(2, 1, 1), mp, p, ws);
  const int grid = std::min(total, wide_sms());
  return launch_pdl(kern, dim3(grid), dim3(wide_threads<EW>()), kSmem, stream, pdl_enabled(), mp, p, ws);
}

// Debug override read once: PI05_WIDE_BN (128 / 256) for STORE / GATED_RESID.
int env_int(const char* name) {
  const char* e = getenv(name);
  return e != nullptr ? atoi(e) : 0;
}

}  // namespace

int wide_choose(int epi, int m_tiles, int n_cols, int kb_total, int sms, int* bn, int* splits, int* pair,
                bool allow_pair) {
  static const int force_bn = env_int("PI05_WIDE_BN");
  static const int force_splits = env_int("PI05_WIDE_SPLITS");
  static const int force_pair = [] {
    const char* e = getenv("PI05_WIDE_PAIR");
    return e != nullptr ? atoi(e) : -1;
  }();
  *splits = 1;
  *pair = 0;
  // CTA pairs pay a longer prologue and (with split-K) a slower epilogue; they win
  // on the long-running projections: gate/up and q|k|v + RoPE at full token tiles
  // (prefix q|k|v 21.1 -> 18.4 us) and long-K ones (the prefix down_proj).
  // PI05_WIDE_PAIR=0 / 1 disables / forces them.
  const bool pair_auto =
      m_tiles >= 4 && (((epi == SK_EPI_GEGLU || epi == SK_EPI_QKV_ROPE) && kb_total >= 16) ||
                       ((epi == SK_EPI_STORE || epi == SK_EPI_GATED_RESID) && kb_total >= 128));
  if (allow_pair && (force_pair > 0 || (force_pair < 0 && pair_auto))) {
    // CTA pairs: 256 x 256 tiles; split-K (STORE / GATED_RESID) until the pairs
    // cover the SMs.
    *bn = 256;
    *pair = 1;
    if (epi == SK_EPI_STORE || epi == SK_EPI_GATED_RESID) {
      const long tiles = (long)((m_tiles + 1) / 2) * ((n_cols + 255) / 256);
      if (force_splits >= 1 && force_splits <= 2)
        *splits = force_splits;
      else if (tiles * 2 <= sms / 2 && kb_total >= 16)
        *splits = 2;
    }
    return 0;
  }
  if (epi == SK_EPI_GEGLU || epi == SK_EPI_QKV_ROPE) {
    *bn = 256;
    return 0;
  }
  // Estimated µs: waves x (k-blocks per tile x time per k-block + fixed cost per
  // tile) + the partial round trip of a split.  A k-block moves 48 KB (256-wide) or
  // 32 KB (128-wide) of operands, at about 100 GB/s per SM.
  double best_cost = 1e30;
  for (int b : {256, 192, 128}) {
    const int nt = (n_cols + b - 1) / b;
    for (int s = 1; s <= 2 && s * 8 <= kb_total; ++s) {
      const long tiles = (long)m_tiles * nt * s;
      const long waves = (tiles + sms - 1) / sms;
      const double kb_per = (double)((kb_total + s - 1) / s);
      // A split adds the partial write + ticket and one L2 round trip per 32
      // columns when the finishing split reads the other partial.
      const double reduce = s > 1 ? 1.0 + 0.9 * (b / 32) : 0.0;
      const double per_kb = b == 256 ? 0.44 : (b == 192 ? 0.39 : 0.34);
      const double cost = (double)waves * (kb_per * per_kb + 3.0) + reduce;
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        *bn = b;
        *splits = s;
      }
    }
  }
  if (force_bn == 128 || force_bn == 192 || force_bn == 256) *bn = force_bn;
  if (force_splits >= 1 && force_splits <= 2) *splits = force_splits;
  // Cluster split-K (*pair = 2): the two K halves of a 128-column tile on the two
  // CTAs of a cluster, which exchange half of their fp32 partials SM to SM and each
  // finish one 64-column slab: no partial round trip through L2, and half the
  // epilogue per CTA.  One tile per cluster, so every tile's pair must fit one wave.
  // PI05_WIDE_CSPLIT=0 disables it.
  static const int force_cs = [] {
    const char* e = getenv("PI05_WIDE_CSPLIT");
    return e != nullptr ? atoi(e) : -1;
  }();
  if (force_cs != 0 && force_bn <= 0 && force_splits <= 0 && (epi == SK_EPI_STORE || epi == SK_EPI_GATED_RESID) &&
      kb_total >= 4 && (kb_total + 1) / 2 <= 40) {
    const long tiles = (long)m_tiles * ((n_cols + 127) / 128);
    if (2 * tiles <= sms) {
      const double cost = (double)((kb_total + 1) / 2) * 0.34 + 3.0 + 1.0;
      if (cost < best_cost - 1e-9) {
        *bn = 128;
        *splits = 2;
        *pair = 2;
      }
    }
  }
  return 0;
}

bool wide_disabled() {
  static int v = [] {
    const char* e = getenv("PI05_WIDE");
    return (e != nullptr && e[0] == '0') ? 1 : 0;
  }();
  return v != 0;
}

int wide_gemm_run(int epi, SkinnyParams p, const void* w0, const void* w1, int w_rows0, int w_rows1, int n_cols,
                  const void* x, int ldx, void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.m_tok <= 0 || p.k <= 0 || p.k % 8 != 0 || n_cols <= 0 || n_cols % 8 != 0) {
    set_last_error("wide_gemm: bad shape m=%d k=%d n=%d", p.m_tok, p.k, n_cols);
    return PI05_ERR_SHAPE;
  }
  if (epi == SK_EPI_QKV_ROPE && (p.head_dim != 256 || p.n_kv_heads != 1)) {
    set_last_error("wide_gemm: QKV+RoPE needs head_dim 256 and one KV head");
    return PI05_ERR_SHAPE;
  }
  WideSched ws;
  const int cta_m_tiles = (p.m_tok + kWBM - 1) / kWBM;
  ws.kb_total = (p.k + kBK - 1) / kBK;
  int bn = 256, splits = 1, pair = 0;
  // The folded LayerNorm runs on single CTAs (its column sums are staged per CTA).
  wide_choose(epi, cta_m_tiles, n_cols, ws.kb_total, wide_sms(), &bn, &splits, &pair, p.ln_colsum == nullptr);
  // Pairs schedule 256-token tiles; every CTA still owns 128 tokens of one.
  const bool csplit = pair == 2;
  if (csplit) pair = 0;
  ws.m_tiles = pair ? (cta_m_tiles + 1) / 2 : cta_m_tiles;
  const int m_tiles_cta = pair ? 2 * ws.m_tiles : ws.m_tiles;
  if (epi == SK_EPI_GEGLU)
    ws.n_tiles = (n_cols + 127) / 128;
  else if (epi == SK_EPI_QKV_ROPE)
    ws.n_tiles = p.n_q_heads + 2 * p.n_kv_heads;
  else
    ws.n_tiles = (n_cols + bn - 1) / bn;
  if (splits > 1 && !csplit) {
    const size_t need = (size_t)m_tiles_cta * ws.n_tiles * splits * kWBM * bn * sizeof(float);
    if (p.accum == nullptr || p.counters == nullptr || need > p.accum_bytes ||
        (long)m_tiles_cta * ws.n_tiles > kWsNormTicketBase || splits > ws.kb_total) {
      splits = 1;
    }
  }
  ws.splits = splits;
  p.splits = splits;
  p.n_valid = n_cols;
  WideMaps mp;
  std::memset(&mp, 0, sizeof(mp));
  int rc = make_tmap_bf16_2d(&mp.x, x, p.m_tok, p.k, ldx, kWBM, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&mp.w0, w0, w_rows0, p.k, p.k, bn / 2, 64, true);
  if (!rc) rc = make_tmap_bf16_2d(&mp.w1, w1, w_rows1, p.k, p.k, bn / 2, 64, true);
  if (rc) return rc;
  if (epi == SK_EPI_QKV_ROPE) {
    const int hd = 256;
    const uint64_t kv_rows = (uint64_t)p.krow0 + p.m_tok;
    rc = make_tmap_bf16_2d(&mp.out, p.q_out, p.m_tok, (uint64_t)p.n_q_heads * hd, (uint64_t)p.n_q_heads * hd, 32,
                           64, true);
    if (!rc) rc = make_tmap_bf16_2d(&mp.in0, p.cos, p.m_tok, hd, hd, 32, 64, true);
    if (!rc) rc = make_tmap_bf16_2d(&mp.in1, p.sin, p.m_tok, hd, hd, 32, 64, true);
    if (!rc) rc = make_tmap_bf16_2d(&mp.kc, p.k_cache, kv_rows, hd, hd, 32, 64, true);
    if (!rc) rc = make_tmap_bf16_2d(&mp.vc, p.v_cache, kv_rows, hd, hd, 32, 64, true);
  } else {
    rc = make_tmap_bf16_2d(&mp.out, p.out, p.m_tok, n_cols, p.ldo, 32, 64, true);
    if (!rc && epi == SK_EPI_GATED_RESID)
      rc = make_tmap_bf16_2d(&mp.in0, p.resid, p.m_tok, n_cols, p.ldr, 32, 64, true);
  }
  if (rc) return rc;
  // Short mainloops (a tile of at most 40 k-blocks) leave the epilogue exposed: give
  // it 8 warps; long ones keep the deeper pipeline.  192-column tiles (three slabs,
  // which 8 warps split unevenly) keep 4 warps and a fourth stage (SigLIP 1.837 ->
  // 1.820 ms).
  const bool wide8 = bn != 192 && (ws.kb_total + ws.splits - 1) / ws.splits <= 40;
  if (csplit) {
    if (epi == SK_EPI_STORE) return wide_launch<SK_EPI_STORE, 128, 3, 8, false, true>(p, ws, mp, st);
    if (epi == SK_EPI_GATED_RESID) return wide_launch<SK_EPI_GATED_RESID, 128, 3, 8, false, true>(p, ws, mp, st);
    set_last_error("wide_gemm: cluster split-K for the row epilogues only");
    return PI05_ERR_INVALID_ARG;
  }
  if (pair) {
    switch (epi) {
      case SK_EPI_STORE:
        return wide8 ? wide_launch<SK_EPI_STORE, 256, 5, 8, true>(p, ws, mp, st)
                     : wide_launch<SK_EPI_STORE, 256, 6, 4, true>(p, ws, mp, st);
      case SK_EPI_GATED_RESID:
        return wide8 ? wide_launch<SK_EPI_GATED_RESID, 256, 5, 8, true>(p, ws, mp, st)
                     : wide_launch<SK_EPI_GATED_RESID, 256, 6, 4, true>(p, ws, mp, st);
      case SK_EPI_GEGLU:
        return wide_launch<SK_EPI_GEGLU, 256, 6, 4, true>(p, ws, mp, st);
      case SK_EPI_QKV_ROPE:
        return wide_launch<SK_EPI_QKV_ROPE, 256, 5, 4, true>(p, ws, mp, st);
      default:
        set_last_error("wide_gemm: unknown epilogue %d", epi);
        return PI05_ERR_INVALID_ARG;
    }
  }
  switch (epi) {
    case SK_EPI_STORE:
      if (wide8) return bn == 256 ? wide_launch<SK_EPI_STORE, 256, 3, 8>(p, ws, mp, st)
                                  : wide_launch<SK_EPI_STORE, 128, 5, 8>(p, ws, mp, st);
      return bn == 256   ? wide_launch<SK_EPI_STORE, 256, 4, 4>(p, ws, mp, st)
             : bn == 192 ? wide_launch<SK_EPI_STORE, 192, 4, 4>(p, ws, mp, st)
                         : wide_launch<SK_EPI_STORE, 128, 6, 4>(p, ws, mp, st);
    case SK_EPI_GATED_RESID:
      if (wide8) return bn == 256 ? wide_launch<SK_EPI_GATED_RESID, 256, 3, 8>(p, ws, mp, st)
                                  : wide_launch<SK_EPI_GATED_RESID, 128, 5, 8>(p, ws, mp, st);
      return bn == 256   ? wide_launch<SK_EPI_GATED_RESID, 256, 4, 4>(p, ws, mp, st)
             : bn == 192 ? wide_launch<SK_EPI_GATED_RESID, 192, 4, 4>(p, ws, mp, st)
                         : wide_launch<SK_EPI_GATED_RESID, 128, 6, 4>(p, ws, mp, st);
    case SK_EPI_GEGLU:
      return wide_launch<SK_EPI_GEGLU, 256, 4, 4>(p, ws, mp, st);
    case SK_EPI_QKV_ROPE:
      return wide_launch<SK_EPI_QKV_ROPE, 256, 3, 4>(p, ws, mp, st);
    default:
      set_last_error("wide_gemm: unknown epilogue %d", epi);
      return PI05_ERR_INVALID_ARG;
  }
}

}  // namespace pi05
