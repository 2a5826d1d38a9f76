// Device-side pieces of the swap-AB tcgen05 GEMM shared by the standalone kernel
// (skinny_gemm.cu) and the persistent denoise kernel (denoise_mega.cu): which
// weight rows form a 128-row tile, how a finished tile is read back (own staging
// tile or the fixed-order sum of split-K partials), and the fused epilogues.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "ptx.cuh"
#include "skinny_gemm.h"

namespace pi05 {
namespace gemm {

constexpr int kBK = 64;           // K elements per stage (one 128-byte swizzle row)
constexpr int kBM = 128;          // UMMA M: weight rows per tile
constexpr int kABytes = kBM * 128;
constexpr int kEpiThreads = 128;  // epilogue threads (four warps, one TMEM lane quarter each)

__device__ __forceinline__ float gelu_tanh_f(float x) {
  // Same op order as the reference's fused epilogue (rlinf_fused_denoise.py:166-172).
  const float t3 = x * 0.5f;
  const float t5 = (x * x) * x;
  const float t8 = x + t5 * 0.044715f;
  const float t11 = tanhf(t8 * 0.7978845608028654f);
  return t3 * (t11 + 1.0f);
}

// The same GELU on the hardware tanh (PTX tanh.approx.f32, one special-function
// instruction, relative error about 2^-11, below the bf16 rounding of the result)
// instead of the accurate tanhf, used where one warp per SM sub-partition must
// evaluate a whole tile (the many-token GEMM epilogue, SigLIP fc1): the
// special-function unit's rate bounds that epilogue.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float t3 = x * 0.5f;
  const float t5 = (x * x) * x;
  const float t8 = x + t5 * 0.044715f;
  return t3 * (tanh_approx(t8 * 0.7978845608028654f) + 1.0f);
}

struct TileRows {
  int row0;  // first row of the low 64-row box (map 0)
  int row1;  // first row of the high 64-row box (map 1)
};

template <int EPI>
__device__ __forceinline__ TileRows tile_rows(const SkinnyParams& p, int tile) {
  TileRows r;
  if (EPI == SK_EPI_GEGLU) {
    r.row0 = tile * 64;
    r.row1 = tile * 64;
  } else if (EPI == SK_EPI_QKV_ROPE) {
    const int half = p.head_dim / 2;
    const int tph = half / 64;  // tiles per rotary head
    const int n_rot_tiles = (p.n_q_heads + p.n_kv_heads) * tph;
    if (tile < n_rot_tiles) {
      const int h = tile / tph, part = tile % tph;
      r.row0 = h * p.head_dim + part * 64;
      r.row1 = r.row0 + half;
    } else {
      r.row0 = (p.n_q_heads + p.n_kv_heads) * p.head_dim + (tile - n_rot_tiles) * kBM;
      r.row1 = r.row0 + 64;
    }
  } else {
    r.row0 = tile * kBM;
    r.row1 = r.row0 + 64;
  }
  return r;
}

// Finished fp32 tile values: either the CTA's own staging tile (no split) or the
// fixed-order sum of every split's partial (split-K).  get8(t, r, v) fills v with
// rows r..r+7 (r % 8 == 0) of token t; tile rows 0..63 come from box 0 and
// 64..127 from box 1.
struct TileSrc {
  const float* st;    // staging tile [TOK][128] (splits == 1)
  const float* part;  // partials [splits][TOK][128] of this tile (splits > 1)
  int splits;
  int tok_stride;     // TOK * 128
  __device__ __forceinline__ void get8(int t, int r, float* v) const {
    if (splits == 1) {
      const float4 a = *reinterpret_cast<const float4*>(st + t * 128 + r);
      const float4 b = *reinterpret_cast<const float4*>(st + t * 128 + r + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      return;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
    const float* q = part + t * 128 + r;
    // Eight splits' loads in flight per pass (one L2 round trip per 8 splits),
    // summed in increasing split order.
    for (int s0 = 0; s0 < splits; s0 += 8) {
      float4 a[8], b[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (s0 + j < splits) {
          a[j] = __ldcg(reinterpret_cast<const float4*>(q + (size_t)(s0 + j) * tok_stride));
          b[j] = __ldcg(reinterpret_cast<const float4*>(q + (size_t)(s0 + j) * tok_stride + 4));
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (s0 + j < splits) {
          v[0] += a[j].x; v[1] += a[j].y; v[2] += a[j].z; v[3] += a[j].w;
          v[4] += b[j].x; v[5] += b[j].y; v[6] += b[j].z; v[7] += b[j].w;
        }
      }
    }
  }
};

// ---------------------------------------------------------------------------
// Split-K through distributed shared memory.  Every split CTA of a tile's cluster
// holds its fp32 partial in its own staging tile (same shared-memory offset in
// every CTA).  After the first cluster barrier, rank r reduces the r-th slice of
// the tile's work units by reading all peers' partials (summed from 0.f in
// increasing rank order, the same order as the global-memory split path) and
// applies the epilogue.  A work unit is 4 consecutive tile rows of one token
// (paired with the same 4 rows + 64 for GEGLU and rotary tiles), so a warp reads
// 512 contiguous bytes of a peer's tile and writes 256 contiguous output bytes.
// The epilogue's global operands for the first pass (residual, gate, bias,
// position rows, cos/sin) are loaded before the barrier, and every split's DSMEM
// load of a pass is issued before the first is consumed: one round trip per pass.
enum ClusterKind { CK_ROWS = 0, CK_GEGLU = 1, CK_ROT = 2, CK_V = 3 };

struct UnitOps {
  float a[4], b[4], c[4], d[4];  // rows: resid/gate/bias/pos; rotary: cos_lo/sin_lo/cos_hi/sin_hi
};

__device__ __forceinline__ void load4bf(const __nv_bfloat16* src, float* f) {
  const uint2 u = *reinterpret_cast<const uint2*>(src);
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) f[j] = __bfloat162float(b[j]);
}

__device__ __forceinline__ void load4f(const float* src, float* f) {
  const float4 a = *reinterpret_cast<const float4*>(src);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
}

// Two fp32 values -> packed bf16 pair (round to nearest even), low half first: one
// paired conversion instruction.
__device__ __forceinline__ uint32_t pack2bf(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ uint2 pack4(const float* f) {
  return make_uint2(pack2bf(f[0], f[1]), pack2bf(f[2], f[3]));
}

// Unit geometry: token t and first tile row r of unit idx (tile-relative).
template <int KIND>
__device__ __forceinline__ void unit_pos(int idx, int& t, int& r) {
  if (KIND == CK_GEGLU || KIND == CK_ROT) {
    t = idx >> 4;
    r = (idx & 15) * 4;
  } else {
    t = idx >> 5;
    r = (idx & 31) * 4;
  }
}

template <int EPI, int KIND>
__device__ __forceinline__ bool unit_valid(const SkinnyParams& p, int tile, int idx, int u1) {
  if (idx >= u1) return false;
  if (KIND == CK_ROWS && p.n_valid > 0) {
    int t, r;
    unit_pos<KIND>(idx, t, r);
    return tile * kBM + r < p.n_valid;
  }
  return true;
}

template <int EPI, int KIND>
__device__ __forceinline__ void unit_load_ops(const SkinnyParams& p, int tile, int tok0, int idx, UnitOps& o) {
  int t, r;
  unit_pos<KIND>(idx, t, r);
  const int tok = tok0 + t;
  if (KIND == CK_ROWS) {
    const int n = tile * kBM + r;
    if (p.bias != nullptr) load4f(p.bias + n, o.c);
    if (EPI == SK_EPI_STORE && p.pos != nullptr) load4f(p.pos + (size_t)(tok % p.pos_rows) * p.ldo + n, o.d);
    if (EPI == SK_EPI_GATED_RESID) {
      load4bf(p.resid + (size_t)tok * p.ldr + n, o.a);
      if (p.gate != nullptr) load4f(p.gate + n, o.b);
    }
  } else if (KIND == CK_ROT) {
    const int hd = p.head_dim, half = hd / 2, tph = half / 64;
    const int dl = (tile % tph) * 64 + r, dh = dl + half;
    load4bf(p.cos + (size_t)tok * hd + dl, o.a);
    load4bf(p.sin + (size_t)tok * hd + dl, o.b);
    load4bf(p.cos + (size_t)tok * hd + dh, o.c);
    load4bf(p.sin + (size_t)tok * hd + dh, o.d);
  }
}

// y[h][j]: the reduced tile values of rows r + 64h + j.  Same arithmetic as
// apply_epilogue for the corresponding epilogue.  Returns, for CK_ROWS, the sum of
// squares of the four bf16 outputs (in order), else 0.
template <int EPI, int KIND>
__device__ __forceinline__ float unit_finish(const SkinnyParams& p, int tile, int tok0, int idx, const UnitOps& o,
                                             const float (&y)[2][4]) {
  int t, r;
  unit_pos<KIND>(idx, t, r);
  const int tok = tok0 + t;
  if (KIND == CK_ROWS) {
    const int n = tile * kBM + r;
    float out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v = y[0][j];
      if (p.bias != nullptr) v += o.c[j];
      if (EPI == SK_EPI_STORE && p.pos != nullptr) v += o.d[j];
      v = bf16_round(v);
      if (EPI == SK_EPI_STORE && p.act == 1) v = gelu_tanh_f(v);
      if (EPI == SK_EPI_GATED_RESID) v = (p.gate != nullptr) ? o.a[j] + v * bf16_round(o.b[j]) : o.a[j] + v;
      out[j] = v;
    }
    *reinterpret_cast<uint2*>(p.out + (size_t)tok * p.ldo + n) = pack4(out);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float b = bf16_round(out[j]);
      ss += b * b;
    }
    return ss;
  } else if (KIND == CK_GEGLU) {
    float out[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = gelu_tanh_f(bf16_round(y[0][j])) * y[1][j];
    *reinterpret_cast<uint2*>(p.out + (size_t)tok * p.ldo + tile * 64 + r) = pack4(out);
  } else if (KIND == CK_ROT) {
    const int hd = p.head_dim, half = hd / 2, tph = half / 64;
    const int h = tile / tph, dl = (tile % tph) * 64 + r, dh = dl + half;
    float olo[4], ohi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float xl = bf16_round(y[0][j]), xh = bf16_round(y[1][j]);
      olo[j] = xl * o.a[j] - xh * o.b[j];
      ohi[j] = xh * o.c[j] + xl * o.d[j];
    }
    __nv_bfloat16* dst = (h < p.n_q_heads) ? p.q_out + ((size_t)tok * p.n_q_heads + h) * hd
                                           : p.k_cache + (size_t)(h - p.n_q_heads) * p.kv_head_stride +
                                                 (size_t)(p.krow0 + tok) * hd;
    *reinterpret_cast<uint2*>(dst + dl) = pack4(olo);
    *reinterpret_cast<uint2*>(dst + dh) = pack4(ohi);
  } else {  // CK_V
    const int hd = p.head_dim;
    const int n_rot_tiles = (p.n_q_heads + p.n_kv_heads) * (hd / 128);
    const int c = (tile - n_rot_tiles) * kBM + r, vh = c / hd, d = c % hd;
    *reinterpret_cast<uint2*>(p.v_cache + (size_t)vh * p.kv_head_stride + (size_t)(p.krow0 + tok) * hd + d) =
        pack4(y[0]);
  }
  return 0.f;
}

// Sum over the 32 lanes of a warp (xor butterfly: the same order on every lane).
__device__ __forceinline__ float warp_sum32(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Row statistics of a CK_ROWS pass: the warp's 32 consecutive units are the 128
// tile rows of one token (unit ranges start on token boundaries), so the warp sum
// of the per-unit sums of squares is that token's partial for this tile.
template <int KIND>
__device__ __forceinline__ void unit_row_ssq(const SkinnyParams& p, int tile, int tok0, int idx, int u1, float ss) {
  if (KIND != CK_ROWS || p.row_ssq == nullptr) return;
  ss = warp_sum32(ss);
  if ((threadIdx.x & 31) == 0 && idx < u1) p.row_ssq[(size_t)tile * p.ssq_ld + tok0 + (idx >> 5)] = ss;
}

// Body of the cluster epilogue for one unit kind and U units per thread per pass.
// Called by all threads of the CTA (it holds the first cluster barrier); `epi`
// selects the 128 epilogue threads, `et` is their index.
template <int EPI, int KIND, int U>
__device__ __forceinline__ void cluster_epilogue_body(const SkinnyParams& p, uint32_t st, int tile, int tok0,
                                                      int u0, int u1, int et, bool epi,
                                                      unsigned long long* stamps) {
  constexpr int H = (KIND == CK_GEGLU || KIND == CK_ROT) ? 2 : 1;
  constexpr int KS = 16 / (U * H) > 0 ? 16 / (U * H) : 1;  // splits per batch of DSMEM loads
  const int splits = p.splits;
  UnitOps ops[U];
  const bool stamp = stamps != nullptr && epi && et == 0;
  if (stamp) stamps[0] = globaltimer_ns();
  // Publish the staging tile, then issue the global operand loads of the first
  // pass while the barrier completes (a release arrive would otherwise wait for
  // them).
  __syncwarp();
  cluster_arrive_release();
  if (epi) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = u0 + u * kEpiThreads + et;
      if (unit_valid<EPI, KIND>(p, tile, idx, u1)) unit_load_ops<EPI, KIND>(p, tile, tok0, idx, ops[u]);
    }
  }
  __syncwarp();
  cluster_wait();
  if (stamp) stamps[1] = globaltimer_ns();
  if (!epi) return;
  for (int base = u0 + et, pass = 0; base < u1; base += U * kEpiThreads, ++pass) {
    bool ok[U];
    uint32_t off[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int idx = base + u * kEpiThreads;
      ok[u] = unit_valid<EPI, KIND>(p, tile, idx, u1);
      int t, r;
      unit_pos<KIND>(idx, t, r);
      off[u] = (uint32_t)(t * kBM + r) * 4u;
      if (pass > 0 && ok[u]) unit_load_ops<EPI, KIND>(p, tile, tok0, idx, ops[u]);
    }
    float acc[U][H][4];
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int h = 0; h < H; ++h)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[u][h][j] = 0.f;
    for (int s0 = 0; s0 < splits; s0 += KS) {
      float4 v[KS][U][H];
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        if (s0 + k < splits) {
          const uint32_t peer = mapa_shared(st, (uint32_t)(s0 + k));
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (ok[u])
#pragma unroll
              for (int h = 0; h < H; ++h) v[k][u][h] = ld_dsmem_f4(peer + off[u] + h * 256u);
        }
      }
#pragma unroll
      for (int k = 0; k < KS; ++k) {
        if (s0 + k < splits) {
#pragma unroll
          for (int u = 0; u < U; ++u)
#pragma unroll
            for (int h = 0; h < H; ++h) {
              acc[u][h][0] += v[k][u][h].x;
              acc[u][h][1] += v[k][u][h].y;
              acc[u][h][2] += v[k][u][h].z;
              acc[u][h][3] += v[k][u][h].w;
            }
        }
      }
    }
    if (stamp && pass == 0) stamps[2] = globaltimer_ns();
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float ss = 0.f;
      if (ok[u]) {
        float y[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int j = 0; j < 4; ++j) y[h][j] = acc[u][h < H ? h : 0][j];
        ss = unit_finish<EPI, KIND>(p, tile, tok0, base + u * kEpiThreads, ops[u], y);
      }
      unit_row_ssq<KIND>(p, tile, tok0, base + u * kEpiThreads, u1, ss);
    }
  }
  if (stamp) stamps[3] = globaltimer_ns();
}

template <int EPI, int KIND>
__device__ __forceinline__ void cluster_epilogue_kind(const SkinnyParams& p, uint32_t st, int tile, int tok0, int mt,
                                                      int rank, int et, bool epi, unsigned long long* stamps) {
  constexpr int H = (KIND == CK_GEGLU || KIND == CK_ROT) ? 2 : 1;
  const int units = mt * (H == 2 ? 16 : 32);
  int u0 = (int)(((long)rank * units) / p.splits);
  int u1 = (int)(((long)(rank + 1) * units) / p.splits);
  if (KIND == CK_ROWS && p.row_ssq != nullptr) {  // whole tokens per rank (row statistics)
    u0 = 32 * ((rank * mt) / p.splits);
    u1 = 32 * (((rank + 1) * mt) / p.splits);
  }
  const int per_thread = (u1 - u0 + kEpiThreads - 1) / kEpiThreads;
  if (per_thread >= 4 && p.splits * H * 4 <= 16)
    cluster_epilogue_body<EPI, KIND, 4>(p, st, tile, tok0, u0, u1, et, epi, stamps);
  else if (per_thread >= 2 && p.splits * H * 2 <= 16)
    cluster_epilogue_body<EPI, KIND, 2>(p, st, tile, tok0, u0, u1, et, epi, stamps);
  else
    cluster_epilogue_body<EPI, KIND, 1>(p, st, tile, tok0, u0, u1, et, epi, stamps);
}

// Whole cluster split-K epilogue (both cluster barriers included); every thread of
// the CTA calls it.  The second barrier keeps each staging tile alive until all
// peers have finished reading it.  `stamps` (optional, shared memory, 5 slots):
// globaltimer before the first barrier, after it, after the first pass's DSMEM
// loads, after the last store, after the exit barrier.
template <int EPI>
__device__ __forceinline__ void cluster_epilogue(const SkinnyParams& p, uint32_t st, int tile, int tok0, int mt,
                                                 int rank, int et, bool epi,
                                                 unsigned long long* stamps = nullptr) {
  if (EPI == SK_EPI_GEGLU) {
    cluster_epilogue_kind<EPI, CK_GEGLU>(p, st, tile, tok0, mt, rank, et, epi, stamps);
  } else if (EPI == SK_EPI_QKV_ROPE) {
    const int n_rot_tiles = (p.n_q_heads + p.n_kv_heads) * (p.head_dim / 128);
    if (tile < n_rot_tiles)
      cluster_epilogue_kind<EPI, CK_ROT>(p, st, tile, tok0, mt, rank, et, epi, stamps);
    else
      cluster_epilogue_kind<EPI, CK_V>(p, st, tile, tok0, mt, rank, et, epi, stamps);
  } else {
    cluster_epilogue_kind<EPI, CK_ROWS>(p, st, tile, tok0, mt, rank, et, epi, stamps);
  }
  // Exit barrier: no CTA leaves while peers still read its staging tile.  The
  // epilogue's global stores need no ordering here, so the arrive is relaxed.
  __syncwarp();
  cluster_arrive_relaxed();
  cluster_wait();
  if (stamps != nullptr && epi && et == 0) stamps[4] = globaltimer_ns();
}

// ---------------------------------------------------------------------------
// Split-K through distributed shared memory, push form.  Rank r of the cluster
// owns tokens [r*mt/splits, (r+1)*mt/splits) of the tile.  As soon as its partial
// is staged, each CTA sends the owner of every other token slice that slice of its
// staging tile with one bulk copy (async proxy, SM-to-SM), completing transaction
// bytes on the owner's barrier `rbar` (armed, and made visible to the cluster by a
// cluster barrier, at kernel start).  The owner waits for its barrier and sums the
// partials from its own shared memory in increasing rank order (0.f + p0 + p1 +
// ..., the order of the pull form and of the global-memory split path), then
// applies the epilogue.  The receive slots are a region of their own: slot s holds
// source s's partial of the owner's token slice, 512 bytes a token.  The exit
// barrier, arrived once a CTA has received everything, keeps every source's
// staging tile alive until all copies out of it have landed.
// Bytes this rank receives in the push form (its token slice from every other rank).
// Receive slot of source split `src` at owner `owner` (src != owner): the owner
// keeps no slot for itself, so splits - 1 slots of its slice cover every source.
__device__ __forceinline__ int recv_slot(int src, int owner) { return src < owner ? src : src - 1; }

__device__ __forceinline__ uint32_t push_recv_bytes(int splits, int mt, int rank) {
  const int t0 = (rank * mt) / splits, t1 = ((rank + 1) * mt) / splits;
  return (uint32_t)((splits - 1) * (t1 - t0) * kBM * 4);
}

template <int EPI, int KIND, int U>
__device__ __forceinline__ void cluster_push_body(const SkinnyParams& p, const float* st, const float* recv,
                                                  uint64_t* rbar, int tile, int tok0, int mt, int rank, int et,
                                                  bool epi, unsigned long long* stamps) {
  constexpr int H = (KIND == CK_GEGLU || KIND == CK_ROT) ? 2 : 1;
  constexpr int UPT = H == 2 ? 16 : 32;  // units per token
  const int splits = p.splits;
  const int t0 = (rank * mt) / splits, t1 = ((rank + 1) * mt) / splits;
  const int u0 = UPT * t0, u1 = UPT * t1;
  const int slot = (t1 - t0) * kBM;  // floats per receive slot
  const bool stamp = stamps != nullptr && epi && et == 0;
  constexpr int kSU = H == 1 ? 4 : 2;  // splits whose loads are in flight together
  UnitOps ops0;  // operands of this thread's first unit, loaded before the receive wait
  if (stamp) stamps[0] = globaltimer_ns();
  bool ok = true;
  if (epi) {
    // The receive slots are this CTA's own (not the ring), armed at kernel start:
    // copy each owner its slice right away.
    if (et < splits && et != rank) {
      const int d0 = (et * mt) / splits, d1 = ((et + 1) * mt) / splits;
      const uint32_t bytes = (uint32_t)(d1 - d0) * kBM * 4u;
      if (bytes > 0)
        bulk_copy_to_peer(mapa_shared(smem_u32(recv) + (uint32_t)recv_slot(rank, et) * bytes, (uint32_t)et),
                          smem_u32(st) + (uint32_t)d0 * kBM * 4u, bytes, mapa_shared(smem_u32(rbar), (uint32_t)et));
    }
    if (stamp) stamps[1] = globaltimer_ns();
    if (unit_valid<EPI, KIND>(p, tile, u0 + et, u1)) unit_load_ops<EPI, KIND>(p, tile, tok0, u0 + et, ops0);
    ok = mbar_wait_cluster(rbar, 0);
    if (!ok) report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
  }
  if (stamp) stamps[2] = globaltimer_ns();
  // Everything this CTA receives has landed: its sources may leave once every
  // owner has said so.
  __syncwarp();
  cluster_arrive_relaxed();
  if (epi && ok) {
    for (int base = u0 + et, pass = 0; base < u1; base += U * kEpiThreads, ++pass) {
      // Rolled: this code runs once per launch and its instruction fetch, not the
      // arithmetic, is what the units wait for when it is unrolled U times.
#pragma unroll 1
      for (int u = 0; u < U; ++u) {
        const int idx = base + u * kEpiThreads;
        float ss = 0.f;
        if (unit_valid<EPI, KIND>(p, tile, idx, u1)) {
          UnitOps o;
          if (pass == 0 && u == 0)
            o = ops0;
          else
            unit_load_ops<EPI, KIND>(p, tile, tok0, idx, o);
          int t, r;
          unit_pos<KIND>(idx, t, r);
          const float* own = st + t * kBM + r;
          const float* rcv = recv + (t - t0) * kBM + r;
          float y[2][4];
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < 4; ++j) y[h][j] = 0.f;
#pragma unroll kSU
          for (int s = 0; s < splits; ++s) {  // loads of kSU splits in flight, sums in split order
            const float* src = s == rank ? own : rcv + recv_slot(s, rank) * slot;
#pragma unroll
            for (int h = 0; h < H; ++h) {
              const float4 v = *reinterpret_cast<const float4*>(src + h * 64);
              y[h][0] += v.x;
              y[h][1] += v.y;
              y[h][2] += v.z;
              y[h][3] += v.w;
            }
          }
          if (H == 1) {
#pragma unroll
            for (int j = 0; j < 4; ++j) y[1][j] = y[0][j];
          }
          ss = unit_finish<EPI, KIND>(p, tile, tok0, idx, o, y);
        }
        unit_row_ssq<KIND>(p, tile, tok0, idx, u1, ss);
      }
    }
  }
  if (stamp) stamps[3] = globaltimer_ns();
  __syncwarp();
  cluster_wait();
  if (stamp) stamps[4] = globaltimer_ns();
}

template <int EPI, int KIND>
__device__ __forceinline__ void cluster_push_kind(const SkinnyParams& p, const float* st, const float* recv,
                                                  uint64_t* rbar, int tile, int tok0, int mt, int rank, int et,
                                                  bool epi, unsigned long long* stamps) {
  constexpr int H = (KIND == CK_GEGLU || KIND == CK_ROT) ? 2 : 1;
  const int tmax = (mt + p.splits - 1) / p.splits;
  const int per_thread = (tmax * (H == 2 ? 16 : 32) + kEpiThreads - 1) / kEpiThreads;
  if (per_thread >= 4)
    cluster_push_body<EPI, KIND, 4>(p, st, recv, rbar, tile, tok0, mt, rank, et, epi, stamps);
  else if (per_thread >= 2)
    cluster_push_body<EPI, KIND, 2>(p, st, recv, rbar, tile, tok0, mt, rank, et, epi, stamps);
  else
    cluster_push_body<EPI, KIND, 1>(p, st, recv, rbar, tile, tok0, mt, rank, et, epi, stamps);
}

// Whole push-form cluster epilogue; every thread of the CTA calls it, the epilogue
// threads after fencing the staging tile they wrote (fence.proxy.async) followed by
// a barrier among themselves.  `recv` must hold (splits - 1) * ceil(mt / splits) *
// 512 bytes (slot recv_slot(s, rank) for source s); `rbar` was initialised with one arrival, armed with push_recv_bytes() and
// published by a cluster barrier before the mainloop.  Trace stamps (optional):
// [0..4] the phases.
template <int EPI>
__device__ __forceinline__ void cluster_push_epilogue(const SkinnyParams& p, const float* st, const float* recv,
                                                      uint64_t* rbar, int tile, int tok0, int mt, int rank, int et,
                                                      bool epi, unsigned long long* stamps) {
  if (EPI == SK_EPI_GEGLU) {
    cluster_push_kind<EPI, CK_GEGLU>(p, st, recv, rbar, tile, tok0, mt, rank, et, epi, stamps);
  } else if (EPI == SK_EPI_QKV_ROPE) {
    const int n_rot_tiles = (p.n_q_heads + p.n_kv_heads) * (p.head_dim / 128);
    if (tile < n_rot_tiles)
      cluster_push_kind<EPI, CK_ROT>(p, st, recv, rbar, tile, tok0, mt, rank, et, epi, stamps);
    else
      cluster_push_kind<EPI, CK_V>(p, st, recv, rbar, tile, tok0, mt, rank, et, epi, stamps);
  } else {
    cluster_push_kind<EPI, CK_ROWS>(p, st, recv, rbar, tile, tok0, mt, rank, et, epi, stamps);
  }
}

// Epilogue items are groups of 8 consecutive tile rows of one token: mt * 16
// groups, or mt * 8 for the epilogues that pair row r with row r + 64.
template <int EPI>
__device__ __forceinline__ int epi_items(const SkinnyParams& p, int tile, int mt) {
  if (EPI == SK_EPI_GEGLU) return mt * 8;
  if (EPI == SK_EPI_QKV_ROPE) {
    const int n_rot_tiles = (p.n_q_heads + p.n_kv_heads) * (p.head_dim / 128);
    return tile < n_rot_tiles ? mt * 8 : mt * 16;
  }
  return mt * 16;
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] = __bfloat162float(b[j]);
}

__device__ __forceinline__ void load8f(const float* src, float* f) {
  const float4 a = *reinterpret_cast<const float4*>(src);
  const float4 b = *reinterpret_cast<const float4*>(src + 4);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

__device__ __forceinline__ uint4 pack8(const float* f) {
  return make_uint4(pack2bf(f[0], f[1]), pack2bf(f[2], f[3]), pack2bf(f[4], f[5]), pack2bf(f[6], f[7]));
}

// Apply the epilogue to item groups [i0, i1).  Each thread handles kBatch
// groups per pass and issues every load of the pass before any store, so the
// global-memory latency of a pass is paid once (outputs may alias inputs, e.g.
// the in-place residual, which rules out compiler reordering across passes).
// KB: groups per pass for a CTA's own staging tile; with split partials each
// group already keeps eight splits' loads in flight, so callers pass KB = 1.
template <int EPI, int KB, class Src>
__device__ __forceinline__ void apply_epilogue(const SkinnyParams& p, const Src& src, int tile, int tok0, int i0,
                                               int i1, int et) {
  constexpr int kBatch = KB;
  if (EPI == SK_EPI_STORE || EPI == SK_EPI_GATED_RESID) {
    constexpr int kBatch = KB < 2 ? KB : 2;  // five 8-float operands per group
    const int n0 = tile * kBM;
    const int n_valid = p.n_valid > 0 ? p.n_valid : 1 << 30;
    for (int base = i0 + et; base < i1; base += kBatch * kEpiThreads) {
      float y[kBatch][8], res[kBatch][8], g[kBatch][8], bi[kBatch][8], ps[kBatch][8];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int idx = base + b * kEpiThreads;
        const int t = idx >> 4, r = (idx & 15) * 8, n = n0 + r, tok = tok0 + t;
        if (idx < i1 && n < n_valid) {
          src.get8(t, r, y[b]);
          if (p.bias != nullptr) load8f(p.bias + n, bi[b]);
          if (EPI == SK_EPI_STORE && p.pos != nullptr) load8f(p.pos + (size_t)(tok % p.pos_rows) * p.ldo + n, ps[b]);
          if (EPI == SK_EPI_GATED_RESID) {
            unpack8(*reinterpret_cast<const uint4*>(p.resid + (size_t)tok * p.ldr + n), res[b]);
            if (p.gate != nullptr) load8f(p.gate + n, g[b]);
          }
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int idx = base + b * kEpiThreads;
        const int t = idx >> 4, r = (idx & 15) * 8, n = n0 + r, tok = tok0 + t;
        float ss = 0.f;
        if (idx < i1 && n < n_valid) {
          float o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float v = y[b][j];
            if (p.bias != nullptr) v += bi[b][j];
            if (EPI == SK_EPI_STORE && p.pos != nullptr) v += ps[b][j];
            v = bf16_round(v);
            if (EPI == SK_EPI_STORE && p.act == 1) v = gelu_tanh_f(v);
            if (EPI == SK_EPI_GATED_RESID) v = (p.gate != nullptr) ? res[b][j] + v * bf16_round(g[b][j]) : res[b][j] + v;
            o[j] = v;
          }
          *reinterpret_cast<uint4*>(p.out + (size_t)tok * p.ldo + n) = pack8(o);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float q = bf16_round(o[j]);
            ss += q * q;
          }
        }
        if (p.row_ssq != nullptr) {
          // Row statistics: the 16 groups of a token are one half-warp (item
          // ranges start on token boundaries when row_ssq is set).
          const unsigned half = 0xffffu << (threadIdx.x & 16);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(half, ss, o);
          if ((threadIdx.x & 15) == 0 && idx < i1) p.row_ssq[(size_t)tile * p.ssq_ld + tok] = ss;
        }
      }
    }
  } else if (EPI == SK_EPI_GEGLU) {
    const int n0 = tile * 64;
    for (int base = i0 + et; base < i1; base += kBatch * kEpiThreads) {
      float gv[kBatch][8], uv[kBatch][8];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int idx = base + b * kEpiThreads;
        if (idx < i1) {
          const int t = idx >> 3, r = (idx & 7) * 8;
          src.get8(t, r, gv[b]);
          src.get8(t, 64 + r, uv[b]);
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int idx = base + b * kEpiThreads;
        if (idx < i1) {
          const int t = idx >> 3, r = (idx & 7) * 8, tok = tok0 + t;
          float o[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = gelu_tanh_f(bf16_round(gv[b][j])) * uv[b][j];
          *reinterpret_cast<uint4*>(p.out + (size_t)tok * p.ldo + n0 + r) = pack8(o);
        }
      }
    }
  } else {  // SK_EPI_QKV_ROPE
    const int hd = p.head_dim, half = hd / 2, tph = half / 64;
    const int n_rot_tiles = (p.n_q_heads + p.n_kv_heads) * tph;
    if (tile < n_rot_tiles) {
      const int h = tile / tph, part = tile % tph;
      constexpr int kRB = KB < 2 ? KB : 2;  // six 8-float operands per group
      for (int base = i0 + et; base < i1; base += kRB * kEpiThreads) {
        float lo[kRB][8], hi[kRB][8], cl[kRB][8], sl[kRB][8], ch[kRB][8], sh[kRB][8];
#pragma unroll
        for (int b = 0; b < kRB; ++b) {
          const int idx = base + b * kEpiThreads;
          if (idx < i1) {
            const int t = idx >> 3, r = (idx & 7) * 8, tok = tok0 + t;
            const int dl = part * 64 + r, dh = dl + half;
            src.get8(t, r, lo[b]);
            src.get8(t, 64 + r, hi[b]);
            unpack8(*reinterpret_cast<const uint4*>(p.cos + (size_t)tok * hd + dl), cl[b]);
            unpack8(*reinterpret_cast<const uint4*>(p.sin + (size_t)tok * hd + dl), sl[b]);
            unpack8(*reinterpret_cast<const uint4*>(p.cos + (size_t)tok * hd + dh), ch[b]);
            unpack8(*reinterpret_cast<const uint4*>(p.sin + (size_t)tok * hd + dh), sh[b]);
          }
        }
#pragma unroll
        for (int b = 0; b < kRB; ++b) {
          const int idx = base + b * kEpiThreads;
          if (idx < i1) {
            const int t = idx >> 3, r = (idx & 7) * 8, tok = tok0 + t;
            const int dl = part * 64 + r, dh = dl + half;
            float olo[8], ohi[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float xl = bf16_round(lo[b][j]), xh = bf16_round(hi[b][j]);
              olo[j] = xl * cl[b][j] - xh * sl[b][j];
              ohi[j] = xh * ch[b][j] + xl * sh[b][j];
            }
            __nv_bfloat16* dst = (h < p.n_q_heads)
                                     ? p.q_out + ((size_t)tok * p.n_q_heads + h) * hd
                                     : p.k_cache + (size_t)(h - p.n_q_heads) * p.kv_head_stride +
                                           (size_t)(p.krow0 + tok) * hd;
            *reinterpret_cast<uint4*>(dst + dl) = pack8(olo);
            *reinterpret_cast<uint4*>(dst + dh) = pack8(ohi);
          }
        }
      }
    } else {
      const int vcol0 = (tile - n_rot_tiles) * kBM;  // column within the packed v heads
      for (int base = i0 + et; base < i1; base += kBatch * kEpiThreads) {
        float v[kBatch][8];
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int idx = base + b * kEpiThreads;
          if (idx < i1) src.get8(idx >> 4, (idx & 15) * 8, v[b]);
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int idx = base + b * kEpiThreads;
          if (idx < i1) {
            const int t = idx >> 4, r = (idx & 15) * 8, tok = tok0 + t;
            const int c = vcol0 + r, vh = c / hd, d = c % hd;
            *reinterpret_cast<uint4*>(p.v_cache + (size_t)vh * p.kv_head_stride + (size_t)(p.krow0 + tok) * hd + d) =
                pack8(v[b]);
          }
        }
      }
    }
  }
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}


}  // namespace gemm
}  // namespace pi05
