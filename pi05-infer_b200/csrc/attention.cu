// Multi-query flash attention with split-KV, for the denoise step (50 suffix
// tokens x 8 heads against P+50 cached keys) and the prefix LM (P tokens x 8
// heads against P keys).
//
// All query heads share the single KV head, so the query rows (token, head) are
// one [R, D] matrix and every CTA of a key range reads its K/V chunk once for 16 x
// W query rows.  The key mask depends only on the key (suffix tokens see every
// valid prefix key and all suffix keys; valid prefix tokens see every valid prefix
// key), so it is a byte per key.
//
// Numerics follow eager_attention_forward (pi05_infer/gemma/modeling_gemma.py:
// 252-275): the score is the bf16-rounded Q.K^T times the scale (rounded again
// to bf16), masked keys are excluded, softmax in fp32 with a running max, the
// probabilities enter P.V as bf16, accumulation in fp32.
//
// mma.sync m16n8k16 (bf16 -> fp32) fragments, ldmatrix from XOR-swizzled shared
// memory, cp.async K/V chunks of 64 keys (double-buffered when a split owns more
// than one chunk).  Chunks of the static part of the cache (the prefix rows, written
// long before) are fetched before the grid-dependency wait, so their latency hides
// behind the previous kernel.  By default two warps share each 16 query rows, one
// taking half the chunk's keys for S and half the head dims for P.V.
//
// Split-KV partials (unnormalised O, running max, sum) go through global memory
// and a second kernel merges them in split order.
#include <cuda_bf16.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "host_util.h"
#include "attention.h"
#include "ptx.cuh"

namespace pi05 {
namespace {

constexpr int kD = 256;           // head dim
constexpr int kChunk = 64;        // keys per chunk
constexpr int kRowBytes = kD * 2; // 512 B per K/V/Q row

// 16-byte chunk c of row r lives at chunk (c ^ (r & 7)) -> conflict-free ldmatrix.
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * kRowBytes + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
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

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16(x)); }

// Exchange area of the warp pairs (H = 2), per row group: both warps' row maxima
// [2][16] floats, their P fragments [2][2 k-steps][4][32 lanes] words, their row
// sums [2][16] floats.
template <int W, int H>
__host__ __device__ constexpr size_t attn_xchg_bytes() {
  return H == 1 ? 0 : (size_t)W * (2 * 16 * 4 + 2 * 2 * 4 * 32 * 4 + 2 * 16 * 4);
}

// Shared memory of one CTA: Q rows, nbuf K and V chunk buffers, the pair exchange
// area, the chunk key masks.
template <int W, int H>
__host__ __device__ constexpr size_t attn_smem_bytes(int nbuf) {
  return (size_t)16 * W * kRowBytes + (size_t)nbuf * 2 * kChunk * kRowBytes + attn_xchg_bytes<W, H>() +
         (size_t)nbuf * kChunk;
}

// W row groups of 16 query rows per CTA, H warps per row group.  With H = 2 the two
// warps of a row group split each chunk: keys [32 hf, 32 hf + 32) for S = Q.K^T and
// head dims [128 hf, 128 hf + 128) for O += P.V.  They agree on the chunk's row max
// and hand each other their P fragments through shared memory (a named barrier of
// the pair for each), and add their row sums at the end.  Each warp then issues half
// the MMAs of a chunk, and an SM runs twice as many warps.
template <int W, int H>
__global__ void __launch_bounds__(W * H * 32, 1)
    mqa_flash_kernel(const AttnParams p) {
  static_assert(H == 1 || H == 2, "one or two warps per row group");
  constexpr int kRows = 16 * W;
  constexpr int kThreads = W * H * 32;
  constexpr int NT = 8 / H;   // 8-key n-tiles of S per warp
  constexpr int DT = 32 / H;  // 8-dim n-tiles of O per warp
  extern __shared__ __align__(128) uint8_t smem[];
  const int nbuf = p.nbuf;
  uint8_t* sQ = smem;                                     // kRows x 512 B
  uint8_t* sK = smem + kRows * kRowBytes;                 // nbuf x 64 x 512 B
  uint8_t* sV = sK + nbuf * kChunk * kRowBytes;           // nbuf x 64 x 512 B
  uint8_t* sX = sV + nbuf * kChunk * kRowBytes;           // pair exchange (H = 2)
  uint8_t* sValid = sX + attn_xchg_bytes<W, H>();         // nbuf x 64 bytes
  float* sMax = reinterpret_cast<float*>(sX);                              // [W][2][16]
  uint32_t* sP = reinterpret_cast<uint32_t*>(sX + W * 2 * 16 * 4);         // [W][2][2][4][32]
  float* sL = reinterpret_cast<float*>(sX + W * (2 * 16 * 4 + 2 * 2 * 4 * 32 * 4));  // [W][2][16]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rg = warp / H, hf = warp % H;
  const int row0 = blockIdx.x * kRows;
  const int split = blockIdx.y;
  // This CTA's observation (blockIdx.z; 0 without a batch).
  const size_t bz = blockIdx.z;
  const __nv_bfloat16* kbase = p.k + bz * p.kv_batch;
  const __nv_bfloat16* vbase = p.v + bz * p.kv_batch;
  const uint8_t* valid_base = p.key_valid + bz * p.valid_batch;
  const bool tr = p.trace != nullptr && tid == 0;
  const uint64_t t_entry = tr ? globaltimer_ns() : 0;
  uint64_t t_wait = 0, t_data = 0, t_loop = 0;
  const int n_chunks_total = (p.kv_len + kChunk - 1) / kChunk;
  const int c_begin = (split * n_chunks_total) / p.splits;
  const int c_end = ((split + 1) * n_chunks_total) / p.splits;

  auto load_chunk = [&](int ci, int buf) {
    const int key0 = ci * kChunk;
    const uint32_t kb = static_cast<uint32_t>(__cvta_generic_to_shared(sK + buf * kChunk * kRowBytes));
    const uint32_t vb = static_cast<uint32_t>(__cvta_generic_to_shared(sV + buf * kChunk * kRowBytes));
    for (int i = tid; i < kChunk * 32; i += kThreads) {
      const int r = i >> 5, c = i & 31;
      const int key = key0 + r;
      const bool ok = key < p.kv_len;
      const size_t off = (size_t)(ok ? key : 0) * p.kv_stride + c * 8;
      cp_async16(kb + swz(r, c), kbase + off, ok);
      cp_async16(vb + swz(r, c), vbase + off, ok);
    }
    for (int r = tid; r < kChunk; r += kThreads) {
      const int key = key0 + r;
      sValid[buf * kChunk + r] = (key < p.kv_len && valid_base[key]) ? 1 : 0;
    }
  };

  // The first chunks' K, V and mask come from the static rows when a whole chunk
  // lies below static_rows: fetch them (one per buffer) before waiting on the
  // previous kernel.
  const bool first_static = c_begin < c_end && (c_begin + 1) * kChunk <= p.static_rows;
  const bool second_static =
      first_static && nbuf == 2 && c_begin + 1 < c_end && (c_begin + 2) * kChunk <= p.static_rows;
  if (first_static) load_chunk(c_begin, 0);
  if (second_static) load_chunk(c_begin + 1, 1);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tr) t_wait = globaltimer_ns();

  // Q rows (zero-fill beyond R).
  for (int i = tid; i < kRows * 32; i += kThreads) {
    const int r = i >> 5, c = i & 31;
    const int gr = row0 + r;
    const bool ok = gr < p.rows;
    cp_async16(static_cast<uint32_t>(__cvta_generic_to_shared(sQ)) + swz(r, c),
               p.q + bz * p.q_batch + (size_t)(ok ? gr : 0) * p.q_stride + c * 8, ok);
  }

  float o[DT][4];
#pragma unroll
  for (int j = 0; j < DT; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};

  if (c_begin < c_end && !first_static) load_chunk(c_begin, 0);
  cp_commit();

  const uint32_t sQa = static_cast<uint32_t>(__cvta_generic_to_shared(sQ));
  const int g = lane >> 2, t4 = lane & 3;
  const float scale = p.scale;
  int scale_exp;
  const bool scale_pow2 = frexpf(scale, &scale_exp) == 0.5f;

  for (int ci = c_begin; ci < c_end; ++ci) {
    const int buf = (ci - c_begin) % nbuf;
    if (ci + 1 < c_end && !(second_static && ci == c_begin)) load_chunk(ci + 1, (buf + 1) % nbuf);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (tr && t_data == 0) t_data = globaltimer_ns();

    const uint32_t sKa = static_cast<uint32_t>(__cvta_generic_to_shared(sK + buf * kChunk * kRowBytes));
    const uint32_t sVa = static_cast<uint32_t>(__cvta_generic_to_shared(sV + buf * kChunk * kRowBytes));

    // S = Q_rg (16 x 256) . K_chunk^T (256 x 64 / H): keys kKeys * hf + j * 8
    constexpr int kKeys = kChunk / H;
    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kD / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      {
        const int r = rg * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(sQa + swz(r, c), a0, a1, a2, a3);
      }
#pragma unroll
      for (int jj = 0; jj < NT / 2; ++jj) {  // two n-tiles of 8 keys per ldmatrix.x4
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3;
        const int r = hf * kKeys + jj * 16 + (mi >> 1) * 8 + (lane & 7);
        const int c = kk * 2 + (mi & 1);
        ldsm_x4(sKa + swz(r, c), b0, b1, b2, b3);
        mma_bf16(s[2 * jj], a0, a1, a2, a3, b0, b1);
        mma_bf16(s[2 * jj + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // scale, mask, online softmax (rows g and g+8 of this row group's 16)
    const uint8_t* valid = sValid + buf * kChunk + hf * kKeys;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      // bf16(bf16(q.k) * scale) two values per conversion (the second rounding is
      // exact, so skipped, for a power-of-two scale); keys j*8 + 2*t4 (+1) of both
      // rows share one 2-byte mask read.
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        bf16_round2(s[j][e], s[j][e + 1]);
        s[j][e] *= scale;
        s[j][e + 1] *= scale;
        if (!scale_pow2) bf16_round2(s[j][e], s[j][e + 1]);
      }
      const uint32_t vk = *reinterpret_cast<const uint16_t*>(valid + j * 8 + 2 * t4);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = ((vk >> ((e & 1) * 8)) & 0xffu) ? s[j][e] : -INFINITY;
        s[j][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffff, mx[h], 2));
    }
    if constexpr (H == 2) {
      // The pair's chunk max: both warps take max(own, partner's) of the same two values.
      float* mine = sMax + (rg * 2 + hf) * 16;
      const float* other = sMax + (rg * 2 + (hf ^ 1)) * 16;
      if (t4 == 0) {
        mine[g] = mx[0];
        mine[g + 8] = mx[1];
      }
      named_bar_sync(1 + rg, 64);
      mx[0] = fmaxf(mx[0], other[g]);
      mx[1] = fmaxf(mx[1], other[g + 8]);
    }
    float corr[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float m_new = fmaxf(m_run[h], mx[h]);
      corr[h] = (m_new == -INFINITY) ? 1.f : __expf(m_run[h] - m_new);
      m_run[h] = m_new;
    }
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int h = e >> 1;
        const float pv = (s[j][e] == -INFINITY) ? 0.f : __expf(s[j][e] - m_run[h]);
        s[j][e] = pv;
        ls[h] += pv;
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ls[h] += __shfl_xor_sync(0xffffffff, ls[h], 1);
      ls[h] += __shfl_xor_sync(0xffffffff, ls[h], 2);
      l_run[h] = l_run[h] * corr[h] + ls[h];
    }
#pragma unroll
    for (int j = 0; j < DT; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // P (16 x 64, bf16) as mma A fragments: k-step kk covers keys 16 kk .. 16 kk + 15
    // (H = 1: packed from s as the P.V loop reaches them).
    uint32_t pa[4][4];
    if constexpr (H == 2) {
      // Each warp holds k-steps 2 hf, 2 hf + 1; the partner's two come through shared
      // memory (lane-contiguous words).  The next chunk's max barrier orders the
      // partner's reads before this warp overwrites its slots.
      uint32_t* mine = sP + (rg * 2 + hf) * (2 * 4 * 32);
      const uint32_t* other = sP + (rg * 2 + (hf ^ 1)) * (2 * 4 * 32);
#pragma unroll
      for (int kl = 0; kl < 2; ++kl) {
        uint32_t w[4];
        w[0] = pack_bf16(s[2 * kl][0], s[2 * kl][1]);
        w[1] = pack_bf16(s[2 * kl][2], s[2 * kl][3]);
        w[2] = pack_bf16(s[2 * kl + 1][0], s[2 * kl + 1][1]);
        w[3] = pack_bf16(s[2 * kl + 1][2], s[2 * kl + 1][3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) mine[(kl * 4 + i) * 32 + lane] = w[i];
      }
      named_bar_sync(1 + rg, 64);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t* src = ((kk >> 1) == hf ? mine : other) + ((kk & 1) * 4) * 32 + lane;
#pragma unroll
        for (int i = 0; i < 4; ++i) pa[kk][i] = src[i * 32];
      }
    }
    // O[:, 256 hf / H ...] += P . V_chunk (64 x 256 / H)
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
      if constexpr (H == 1) {
        pa[kk][0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
        pa[kk][1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
        pa[kk][2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[kk][3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      }
#pragma unroll
      for (int jj = 0; jj < DT / 2; ++jj) {  // two 8-wide d tiles per ldmatrix.x4.trans
        uint32_t b0, b1, b2, b3;
        const int mi = lane >> 3;
        const int r = kk * 16 + (mi & 1) * 8 + (lane & 7);
        const int c = hf * DT + jj * 2 + (mi >> 1);
        ldsm_x4_t(sVa + swz(r, c), b0, b1, b2, b3);
        mma_bf16(o[2 * jj], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
        mma_bf16(o[2 * jj + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  if (tr) t_loop = globaltimer_ns();
  // Trace record {tag << 32 | smid << 16 | cta, entry, grid-dependency wait done,
  // first chunk ready, key loop done, output / partial written, 0, 0}.
  auto trace_out = [&]() {
    if (!tr) return;
    const unsigned long long slot = atomicAdd(p.trace, 1ull);
    if (slot < p.trace[1]) {
      unsigned long long* w = p.trace + 8 + slot * 8;
      w[0] = ((unsigned long long)p.trace_tag << 32) | ((unsigned long long)smid() << 16) |
             (blockIdx.y * gridDim.x + blockIdx.x);
      w[1] = t_entry;
      w[2] = t_wait;
      w[3] = t_data;
      w[4] = t_loop;
      w[5] = globaltimer_ns();
      w[6] = 0;
      w[7] = 0;
    }
  };

  if constexpr (H == 2) {
    // Row sums of the pair, added in key order (warp 0's keys first).
    float* mine = sL + (rg * 2 + hf) * 16;
    if (t4 == 0) {
      mine[g] = l_run[0];
      mine[g + 8] = l_run[1];
    }
    named_bar_sync(1 + rg, 64);
    const float* l0 = sL + rg * 2 * 16;
    l_run[0] = l0[g] + l0[16 + g];
    l_run[1] = l0[g + 8] + l0[16 + g + 8];
  }
  // Output: rows (rg*16 + g) and (+8), columns hf*256/H + j*8 + 2*t4 .. +1.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = row0 + rg * 16 + g + h * 8;
    if (r >= p.rows) continue;
    const int col0 = hf * (kD / H);
    if (p.splits == 1) {
      const float inv = l_run[h] > 0.f ? 1.f / l_run[h] : 0.f;
      __nv_bfloat16* dst = p.out + bz * p.out_batch + (size_t)r * p.out_stride + col0;
#pragma unroll
      for (int j = 0; j < DT; ++j) {
        *reinterpret_cast<__nv_bfloat162*>(dst + j * 8 + 2 * t4) =
            __floats2bfloat162_rn(o[j][2 * h] * inv, o[j][2 * h + 1] * inv);
      }
    } else {
      float* dst = p.part_o + (((size_t)bz * p.splits + split) * p.part_rows + r) * kD + col0;
#pragma unroll
      for (int j = 0; j < DT; ++j)
        *reinterpret_cast<float2*>(dst + j * 8 + 2 * t4) = make_float2(o[j][2 * h], o[j][2 * h + 1]);
      if (t4 == 0 && hf == 0) {
        p.part_ml[(((size_t)bz * p.splits + split) * p.part_rows + r) * 2] = m_run[h];
        p.part_ml[(((size_t)bz * p.splits + split) * p.part_rows + r) * 2 + 1] = l_run[h];
      }
    }
  }
  trace_out();
}

// One warp per row: merge the split partials (O unnormalised, running max m,
// sum l).  Lane s holds split s's (m, l); each lane owns 8 columns.  Every load of
// the row (all splits' O columns and the (m, l) pairs) is issued before the first is
// consumed, so the merge costs one L2 round trip.
constexpr int kCombineMaxSplits = 16;

__global__ void __launch_bounds__(64) mqa_combine_kernel(const AttnParams p) {
  const bool tr = p.trace != nullptr && threadIdx.x == 0;
  const uint64_t t_entry = tr ? globaltimer_ns() : 0;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const uint64_t t_wait = tr ? globaltimer_ns() : 0;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  // Trace record {(tag + 1) << 32 | cta, entry, grid-dependency wait done, this
  // thread's row written, 0, 0, 0, 0}.
  auto trace_out = [&]() {
    if (!tr) return;
    const unsigned long long slot = atomicAdd(p.trace, 1ull);
    if (slot < p.trace[1]) {
      unsigned long long* w = p.trace + 8 + slot * 8;
      w[0] = ((unsigned long long)(p.trace_tag + 1) << 32) | blockIdx.x;
      w[1] = t_entry;
      w[2] = t_wait;
      w[3] = globaltimer_ns();
      w[4] = w[5] = w[6] = w[7] = 0;
    }
  };
  if (warp >= p.rows) {
    trace_out();
    return;
  }
  const int r = warp;
  // Observation blockIdx.y: its partials and output rows.
  const size_t bz = blockIdx.y;
  const float* part_o = p.part_o + bz * p.splits * p.part_rows * kD;
  const float* part_ml = p.part_ml + bz * p.splits * p.part_rows * 2;
  float ms = -INFINITY, ls = 0.f;
  if (lane < p.splits) {
    ms = part_ml[((size_t)lane * p.part_rows + r) * 2];
    ls = part_ml[((size_t)lane * p.part_rows + r) * 2 + 1];
  }
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (p.splits <= kCombineMaxSplits) {
    float4 a[kCombineMaxSplits], b[kCombineMaxSplits];
#pragma unroll
    for (int j = 0; j < kCombineMaxSplits; ++j) {
      if (j < p.splits) {
        const float4* src = reinterpret_cast<const float4*>(part_o + ((size_t)j * p.part_rows + r) * kD + lane * 8);
        a[j] = __ldcg(src);
        b[j] = __ldcg(src + 1);
      }
    }
    float mmax = ms;
    for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffff, mmax, o));
    const float w = (lane < p.splits && ms != -INFINITY) ? __expf(ms - mmax) : 0.f;
    float l = ls * w;
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffff, l, o);
#pragma unroll
    for (int j = 0; j < kCombineMaxSplits; ++j) {
      if (j < p.splits) {
        const float wj = __shfl_sync(0xffffffff, w, j);
        acc[0] += a[j].x * wj; acc[1] += a[j].y * wj; acc[2] += a[j].z * wj; acc[3] += a[j].w * wj;
        acc[4] += b[j].x * wj; acc[5] += b[j].y * wj; acc[6] += b[j].z * wj; acc[7] += b[j].w * wj;
      }
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= inv;
  } else {
    float mmax = ms;
    for (int o = 16; o > 0; o >>= 1) mmax = fmaxf(mmax, __shfl_xor_sync(0xffffffff, mmax, o));
    const float w = (lane < p.splits && ms != -INFINITY) ? __expf(ms - mmax) : 0.f;
    float l = ls * w;
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffff, l, o);
    for (int j = 0; j < p.splits; ++j) {
      const float wj = __shfl_sync(0xffffffff, w, j & 31);
      const float4* src = reinterpret_cast<const float4*>(part_o + ((size_t)j * p.part_rows + r) * kD + lane * 8);
      const float4 x = __ldcg(src), y = __ldcg(src + 1);
      acc[0] += x.x * wj; acc[1] += x.y * wj; acc[2] += x.z * wj; acc[3] += x.w * wj;
      acc[4] += y.x * wj; acc[5] += y.y * wj; acc[6] += y.z * wj; acc[7] += y.w * wj;
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= inv;
  }
  __nv_bfloat16* dst = p.out + bz * p.out_batch + (size_t)r * p.out_stride + lane * 8;
  uint4 pk;
  pk.x = pack_bf16(acc[0], acc[1]);
  pk.y = pack_bf16(acc[2], acc[3]);
  pk.z = pack_bf16(acc[4], acc[5]);
  pk.w = pack_bf16(acc[6], acc[7]);
  *reinterpret_cast<uint4*>(dst) = pk;
  trace_out();
}

}  // namespace

namespace {

template <int W, int H>
int set_attn_smem() {
  static bool done[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && done[dev]) return PI05_OK;
  cudaError_t e = cudaFuncSetAttribute(mqa_flash_kernel<W, H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)attn_smem_bytes<W, H>(2));
  if (e != cudaSuccess) {
    set_last_error("attention smem attr: %s", cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  if (dev < 16) done[dev] = true;
  return PI05_OK;
}

}  // namespace

// Query rows above which the tcgen05 kernel is used (PI05_ATTN_TC_MIN_ROWS overrides,
// for tuning).
int tc_min_rows() {
  static int v = [] {
    const char* e = getenv("PI05_ATTN_TC_MIN_ROWS");
    return e != nullptr ? atoi(e) : 1024;
  }();
  return v;
}

// Two rows (warps) per CTA, so the partial reads spread over every SM.
int launch_combine(const AttnParams& p, cudaStream_t st) {
  return launch_pdl(mqa_combine_kernel, dim3((p.rows + 1) / 2, p.batch), dim3(64), 0, st, pdl_enabled(), p);
}

// mma.sync path: W row groups of 16 query rows per CTA, H warps per row group
// (default W = 2, H = 2; PI05_ATTN_WARPS=4 selects W = 4, PI05_ATTN_PAIR=0 H = 1,
// for tuning).
template <int W, int H>
int mma_sync_attention(AttnParams p, float* part, size_t part_bytes, int splits, cudaStream_t st) {
  constexpr int kRows = 16 * W;
  const int row_blocks = (p.rows + kRows - 1) / kRows;
  const int n_chunks = (p.kv_len + kChunk - 1) / kChunk;
  int sms = 148;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  static const int force_splits = [] {
    const char* e = getenv("PI05_ATTN_SPLITS");
    return e != nullptr ? atoi(e) : 0;
  }();
  if (splits <= 0 && force_splits > 0) splits = force_splits;  // tuning
  const bool auto_splits = splits <= 0;
  if (auto_splits) {
    // Single warps: up to two CTAs per SM (a CTA's 2 warps use half of the SM's
    // sub-partitions; the key loop is bound by the mma.sync rate per sub-partition).
    // Warp pairs: up to one CTA per SM, so a split of the denoise owns two chunks
    // and loads the second during the first (682 vs 694 us/step with 16 splits).
    const int per_sm = H == 2 ? 1 : 2;
    splits = 1;
    while (row_blocks * p.batch * splits * 2 <= per_sm * sms && splits * 2 <= n_chunks) splits *= 2;
  }
  splits = splits > n_chunks ? n_chunks : splits;
  splits = splits > 32 ? 32 : splits;
  p.splits = splits;
  p.nbuf = (n_chunks + splits - 1) / splits > 1 ? 2 : 1;
  const size_t smem = attn_smem_bytes<W, H>(p.nbuf);
  if (splits > 1) {
    const size_t need_o = (size_t)p.batch * splits * p.rows * kD * sizeof(float);
    const size_t need = need_o + (size_t)p.batch * splits * p.rows * 2 * sizeof(float);
    if (part == nullptr || need > part_bytes) {
      set_last_error("attention: workspace too small (%zu needed)", need);
      return PI05_ERR_WORKSPACE;
    }
    p.part_rows = p.rows;
    p.part_o = part;
    p.part_ml = part + (size_t)p.batch * splits * p.rows * kD;
  }
  int rc = set_attn_smem<W, H>();
  if (rc) return rc;
  rc = launch_pdl(mqa_flash_kernel<W, H>, dim3(row_blocks, splits, p.batch), dim3(W * H * 32), smem, st,
                  pdl_enabled(), p);
  if (rc || splits == 1) return rc;
  return launch_combine(p, st);
}

int mqa_attention_run(AttnParams p, float* part, size_t part_bytes, int splits, void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.head_dim != kD) {
    set_last_error("attention: head_dim %d unsupported (256 only)", p.head_dim);
    return PI05_ERR_SHAPE;
  }
  if (p.rows <= 0 || p.kv_len <= 0 || p.batch <= 0 || p.batch > 65535) {
    set_last_error("attention: empty rows/keys or bad batch");
    return PI05_ERR_SHAPE;
  }
  // tcgen05 for many query rows (prefix LM: 968 x 8); the mma.sync kernel below is
  // faster for the denoise suffix (50 x 8 rows), where each CTA owns one key chunk.
  if (tc_attention_enabled() && p.rows > tc_min_rows() && p.batch == 1)
    return mqa_tc_attention_run(p, part, part_bytes, splits, st, launch_combine);
  static const int warps = [] {
    const char* e = getenv("PI05_ATTN_WARPS");
    return (e != nullptr && atoi(e) == 4) ? 4 : 2;
  }();
  static const bool pair = [] {
    const char* e = getenv("PI05_ATTN_PAIR");
    return e == nullptr || atoi(e) != 0;
  }();
  if (warps == 4) return pair ? mma_sync_attention<4, 2>(p, part, part_bytes, splits, st)
                              : mma_sync_attention<4, 1>(p, part, part_bytes, splits, st);
  return pair ? mma_sync_attention<2, 2>(p, part, part_bytes, splits, st)
              : mma_sync_attention<2, 1>(p, part, part_bytes, splits, st);
}

}  // namespace pi05
