// Swap-AB tcgen05 GEMM for the denoise step's small-token projections.
//
//   Y[t, n] = sum_k X[t, k] * W[n, k]       (X: tokens x K activations, W: N x K weights)
//
// is computed as Y^T = W * X^T so that the weights fill the 128-row UMMA M
// dimension and the (<= 64 .. 256) tokens form the UMMA N dimension.  Weights
// stream from HBM by TMA (128-byte swizzle, evict-first) into a STAGES-deep ring;
// one elected thread issues tcgen05.mma into a TMEM accumulator; four epilogue
// warps read TMEM back and apply the fused epilogue.
//
// A 128-row A tile is assembled from two 64-row TMA boxes, which lets one tile pair
// rows that the epilogue must combine without re-packing the reference's weights:
//   * GEGLU     : 64 rows of W_gate + the same 64 rows of W_up       (gelu_tanh(g)*u)
//   * QKV_ROPE  : rows d..d+63 and d+D/2..d+D/2+63 of one head        (RoPE pairs)
//   * STORE / GATED_RESID : 128 consecutive rows.
//
// Split-K: when N has too few 128-row tiles to cover the SMs, the K range is split
// across CTAs.  Each split stores its fp32 partial in the workspace, the splits of
// a tile meet at a bounded counter barrier, and each then reduces 1/splits of the
// tile in fixed split order and applies the epilogue to that slice, so results
// do not depend on CTA timing.
//
// Reference ops replaced (pi05_infer/gemma/rlinf_fused_denoise.py):
//   gate_up_geglu  (:350-389, kernel :116-180)
//   qkv_rope_kv    (:392-467, kernel :182-332)
// and the o_proj / down_proj GEMMs with _gated_residual
// (pi05_infer/gemma/modeling_gemma.py:231-249, :455-456, :138-148, :503).
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "elementwise.h"
#include "gemm_epilogue.cuh"
#include "host_util.h"
#include "ptx.cuh"
#include "skinny_gemm.h"
#include "wide_gemm.h"

namespace pi05 {

namespace {

using namespace gemm;
constexpr int kThreads = 192;     // warp0 TMA, warp1 MMA/TMEM, warps2-5 epilogue
// Dedicated receive slots of the push-form split-K (64-token tile only): at most
// (splits - 1) * ceil(tokens / splits) rows of 512 bytes; the launcher checks.
template <int TOK>
constexpr int recv_bytes() {
  return TOK == 64 ? 32768 : 0;
}

// Folded-norm area: rstd per token and the folded bias of the tile's rows.
template <int TOK>
constexpr int fold_bytes() {
  return TOK * 4 + kBM * 4;
}

// Ring, barrier area (512 B), receive slots; the folded-norm area follows and is
// only allocated for launches with a folded norm.
template <int TOK, int STAGES>
constexpr int smem_base_bytes() {
  return 1024 + STAGES * (kABytes + TOK * 128) + 512 + recv_bytes<TOK>();
}

template <int TOK, int STAGES>
constexpr int smem_bytes() {
  return smem_base_bytes<TOK, STAGES>() + fold_bytes<TOK>();
}

// Small-token variants are limited to 170 registers so that two CTAs fit per SM:
// with PDL the next kernel's CTAs then become resident (and start their weight
// prefetch) while this kernel's CTAs are still finishing.  This matters most for
// q|k|v, whose CTAs otherwise cannot share an SM with a down_proj CTA and start
// only as down_proj's CTAs exit (1.6 µs of launch spread per layer on B200).
template <int EPI, int TOK, int STAGES>
__global__ void __launch_bounds__(kThreads, (TOK <= 128 ? 2 : 1))
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap tm_w0, const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_x, const SkinnyParams p) {
  constexpr int kBBytes = TOK * 128;
  constexpr int kStageBytes = kABytes + kBBytes;
  constexpr uint32_t kTmemCols = TOK < 32 ? 32 : TOK;
  constexpr uint32_t kIdesc = umma_idesc_bf16(kBM, TOK);
  static_assert(TOK % 16 == 0 && TOK >= 16 && TOK <= 256, "UMMA N for M=128");
  static_assert(TOK * kBM * 4 <= STAGES * kStageBytes, "epilogue staging must fit in the ring");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  unsigned long long* s_stamp = reinterpret_cast<unsigned long long*>(accum + 1);  // 8-byte aligned
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accum + 2);
  int* s_flag = reinterpret_cast<int*>(s_tmem + 1);  // [0] abort, [1] ticket
  uint64_t* rbar = accum + 9;                         // push-form split-K: partial slices received
  float* recv = reinterpret_cast<float*>(smem + STAGES * kStageBytes + 512);     // push-form receive slots
  // Folded norm of X (gate/up, q|k|v; 64-token tile): rstd per token and the bias
  // of the tile's 128 rows.
  constexpr bool kFoldCapable = TOK == 64 && (EPI == SK_EPI_GEGLU || EPI == SK_EPI_QKV_ROPE);
  const bool fold = kFoldCapable && p.fold_ssq != nullptr;
  float* s_rstd = recv + recv_bytes<TOK>() / 4;  // [TOK]
  float* s_fbias = s_rstd + TOK;                 // [kBM]
  float* stage_tile = reinterpret_cast<float*>(smem);
  constexpr bool kPushFits = recv_bytes<TOK>() > 0;
  const bool push = kPushFits && p.cluster && p.push;

  const uint64_t t_entry = (p.trace != nullptr) ? globaltimer_ns() : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
  const int tok0 = blockIdx.y * TOK;
  const int mt = min(TOK, p.m_tok - tok0);
  const int kb0 = (split * p.kb_total) / p.splits;
  const int kb1 = ((split + 1) * p.kb_total) / p.splits;
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    mbar_init(rbar, 1);
    s_flag[0] = 0;
    s_flag[1] = 0;
    fence_mbar_init();
    // Push form: expect this rank's token slice from every other split.
    if (push) mbar_arrive_expect_tx(rbar, push_recv_bytes(p.splits, mt, (int)cluster_ctarank()));
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_w0);
    prefetch_tmap(&tm_w1);
    prefetch_tmap(&tm_x);
  }
  if (warp == 1) {
    tmem_alloc(s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if (push) {
    // Every receive barrier of the cluster is armed before any CTA can copy into
    // it (a peer copies as soon as its own partial is staged).
    cluster_arrive_release();
    cluster_wait();
  }
  tc_fence_after();
  const uint32_t tmem_acc = *s_tmem;
  const uint64_t t_start = (p.trace != nullptr) ? globaltimer_ns() : 0;
  uint64_t t_pdl = 0, t_acc = 0, t_pub = 0, t_red = 0;
  uint64_t t_staged = 0, t_bar = 0;  // accumulator staged in shared memory; epilogue barrier passed
  // Let the next kernel in the stream start its prologue / weight prefetch.
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      const TileRows tr = tile_rows<EPI>(p, tile);
      const int pre = min(STAGES, nk);
      // Weights do not depend on the previous kernel: issue them before the grid-dependency wait.
      if (p.trace != nullptr) s_stamp[0] = globaltimer_ns();
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], kStageBytes);
        const int kx = (kb0 + i) * kBK;
        tma_load_2d(sA + i * kABytes, &tm_w0, &full[i], kx, tr.row0, pol_w);
        tma_load_2d(sA + i * kABytes + kABytes / 2, &tm_w1, &full[i], kx, tr.row1, pol_w);
      }
      // The k-blocks past the ring are loaded only once MMAs free a stage: bring
      // their weights into L2 now, so those loads do not wait on HBM.
      for (int i = pre; i < nk && i < pre + 8; ++i) {
        const int kx = (kb0 + i) * kBK;
        tma_prefetch_2d(&tm_w0, kx, tr.row0);
        tma_prefetch_2d(&tm_w1, kx, tr.row1);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) tma_load_2d(sB + i * kBBytes, &tm_x, &full[i], (kb0 + i) * kBK, tok0, pol_x);
      for (int i = pre; i < nk; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1)) {
          report_status(p.status, PI05_DEV_TIMEOUT_PRODUCER);
          s_flag[0] = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        const int kx = (kb0 + i) * kBK;
        tma_load_2d(sA + s * kABytes, &tm_w0, &full[s], kx, tr.row0, pol_w);
        tma_load_2d(sA + s * kABytes + kABytes / 2, &tm_w1, &full[s], kx, tr.row1, pol_w);
        tma_load_2d(sB + s * kBBytes, &tm_x, &full[s], kx, tok0, pol_x);
      }
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      bool ok = true;
      for (int i = 0; i < nk && ok; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
          report_status(p.status, PI05_DEV_TIMEOUT_MMA);
          s_flag[0] = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * kABytes);
        const uint32_t b0 = smem_u32(sB + s * kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          umma_bf16(tmem_acc, umma_sdesc_sw128(a0 + kk * 32), umma_sdesc_sw128(b0 + kk * 32), kIdesc,
                    (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(accum);
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter = warp % 4.
    if constexpr (kFoldCapable) {
      if (fold) {
        // The folded bias is a weight: staged before the grid-dependency wait.
        const TileRows tr = tile_rows<EPI>(p, tile);
        const int i = threadIdx.x - 64;
        s_fbias[i] = split != 0 ? 0.f : (i < 64 ? p.fold_bias0[tr.row0 + i] : p.fold_bias1[tr.row1 + i - 64]);
      }
    }
    pdl_wait();
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int et = threadIdx.x - 64;
    if (p.trace != nullptr) t_pdl = globaltimer_ns();
    if constexpr (kFoldCapable) {
      if (fold) {
        // rstd of token et from the producer's partial sums of squares (in order);
        // these loads overlap the X load and the MMAs.
        if (et < TOK) {
          float ssv[kNormMaxParts];
#pragma unroll
          for (int j = 0; j < kNormMaxParts; ++j)
            ssv[j] = (et < mt && j < p.fold_parts) ? __ldcg(p.fold_ssq + (size_t)j * p.fold_ld + tok0 + et) : 0.f;
          float ss = 0.f;
#pragma unroll
          for (int j = 0; j < kNormMaxParts; ++j) ss += ssv[j];
          s_rstd[et] = et < mt ? rsqrtf(ss / (float)p.fold_d + p.fold_eps) : 0.f;
        }
        named_bar_sync(1, kEpiThreads);  // s_rstd, s_fbias
      }
    }
    const bool ok = mbar_wait(accum, 0);
    if (!ok) report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
    if (p.trace != nullptr) t_acc = globaltimer_ns();
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < TOK / 32; ++c) {
        float v[32];
        tmem_ld32(tmem_acc + ((uint32_t)(q * 32) << 16) + c * 32, v);
        if constexpr (kFoldCapable) {
          if (fold) {  // each split scales its partial; split 0 adds the bias
            const float fb = s_fbias[row];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaf(v[j], s_rstd[c * 32 + j], fb);
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) stage_tile[(c * 32 + j) * kBM + row] = v[j];
      }
    }
    if (p.trace != nullptr) t_staged = globaltimer_ns();
    if (push) fence_proxy_async_smem();  // the bulk copies read the staging tile
    named_bar_sync(1, kEpiThreads);
    if (p.trace != nullptr) t_bar = globaltimer_ns();
    const int items = epi_items<EPI>(p, tile, mt);
    if (ok && p.splits == 1) {
      TileSrc src{stage_tile, nullptr, 1, TOK * kBM};
      apply_epilogue<EPI, 4>(p, src, tile, tok0, 0, items, et);
    } else if (ok && !p.cluster) {
      // Deterministic split-K: publish this split's partial, wait (bounded) until
      // every split of the tile has published, then reduce a 1/splits slice of the
      // tile in fixed split order and apply the epilogue to it.  All CTAs of the
      // grid are co-resident (the launcher keeps split grids within one wave).
      const size_t tile_id = (size_t)blockIdx.y * p.n_tiles + tile;
      float* part = p.accum + tile_id * p.splits * TOK * kBM;
      float* mine = part + (size_t)split * TOK * kBM;
      // Test hook: this split of tile 0 leaves its partial and arrival out.
      const bool skip = p.fault_skip_split == split && tile_id == 0;
      if (!skip)
        for (int idx = et * 4; idx < mt * kBM; idx += kEpiThreads * 4)
          __stcg(reinterpret_cast<float4*>(mine + idx),
                 make_float4(stage_tile[idx], stage_tile[idx + 1], stage_tile[idx + 2], stage_tile[idx + 3]));
      __threadfence();
      named_bar_sync(1, kEpiThreads);
      if (p.trace != nullptr) t_pub = globaltimer_ns();
      int* arrive = p.counters + 2 * tile_id;
      int* depart = arrive + 1;
      if (et == 0) {
        if (!skip) atomicAdd(arrive, 1);
        int seen = ld_acquire(arrive);
        if (seen < p.splits) {
          const uint64_t t0 = globaltimer_ns();
          const uint64_t limit = p.wait_ns != 0 ? p.wait_ns : kWaitTimeoutNs;
          while ((seen = ld_acquire(arrive)) < p.splits) {
            if (globaltimer_ns() - t0 > limit) {
              report_status(p.status, PI05_DEV_TIMEOUT_EPILOGUE);
              break;
            }
          }
        }
        s_flag[1] = (seen >= p.splits) ? 1 : 0;
      }
      named_bar_sync(1, kEpiThreads);
      if (s_flag[1]) {
        __threadfence();
        TileSrc src{nullptr, part, p.splits, TOK * kBM};
        int i0 = (int)(((long)split * items) / p.splits);
        int i1 = (int)(((long)(split + 1) * items) / p.splits);
        if (p.row_ssq != nullptr) {  // whole tokens per split (row statistics)
          i0 = 16 * ((split * mt) / p.splits);
          i1 = 16 * (((split + 1) * mt) / p.splits);
        }
        apply_epilogue<EPI, 1>(p, src, tile, tok0, i0, i1, et);
      }
      named_bar_sync(1, kEpiThreads);
      if (et == 0 && atomicAdd(depart, 1) == p.splits - 1) {
        // Last one out: re-arm the tile's counters for the next launch.
        atomicExch(arrive, 0);
        atomicExch(depart, 0);
      }
    }
  }

  // Cluster split-K: every split CTA of the tile has its partial in its staging
  // tile; cluster_epilogue reduces this rank's slice through DSMEM and applies the
  // epilogue between its two cluster barriers.
  unsigned long long* cl_stamps = reinterpret_cast<unsigned long long*>(accum + 4);  // [5]
  if (p.cluster) {
    __syncwarp();
    if (push)
      cluster_push_epilogue<EPI>(p, stage_tile, recv, rbar, tile, tok0, mt, (int)cluster_ctarank(),
                                 (int)threadIdx.x - 64, warp >= 2, p.trace != nullptr ? cl_stamps : nullptr);
    else
      cluster_epilogue<EPI>(p, smem_u32(stage_tile), tile, tok0, mt, (int)cluster_ctarank(), (int)threadIdx.x - 64,
                            warp >= 2, p.trace != nullptr ? cl_stamps : nullptr);
    if (p.trace != nullptr) {
      t_red = globaltimer_ns();
      t_pub = cl_stamps[1];  // written by this thread (epilogue thread 0) after the first cluster barrier
    }
  }

  if (p.trace != nullptr && threadIdx.x == 64) {
    const unsigned long long cta = ((unsigned long long)smid() << 16) | (blockIdx.y * gridDim.x + blockIdx.x);
    const unsigned long long slot = atomicAdd(p.trace, p.cluster ? 2ull : 1ull);
    const unsigned long long cap = p.trace[1];  // records the buffer holds
    if (slot < cap) {
      unsigned long long* w = p.trace + 8 + slot * 8;
      w[0] = ((unsigned long long)p.trace_tag << 32) | cta;
      w[1] = t_entry;
      w[2] = t_start;
      w[3] = t_pdl;
      w[4] = t_acc;
      w[5] = t_pub;
      w[6] = t_red != 0 ? t_red : globaltimer_ns();
      w[7] = s_stamp[0];
    }
    if (p.cluster && slot + 1 < cap) {
      // Cluster epilogue record (tag + 2^30): before / after the first cluster
      // barrier (push form: epilogue start / copies issued), first DSMEM pass
      // summed (push form: slices received), last store issued, exit barrier passed,
      // then the accumulator staged in shared memory and the epilogue barrier passed.
      unsigned long long* w = p.trace + 8 + (slot + 1) * 8;
      w[0] = ((unsigned long long)(p.trace_tag + (1 << 30)) << 32) | cta;
      for (int i = 0; i < 5; ++i) w[1 + i] = cl_stamps[i];
      w[6] = t_staged;
      w[7] = t_bar;
    }
  }

  // Teardown.  If the producer bailed out, the ring may still have copies in
  // flight: wait (bounded) for every armed stage before releasing shared memory.
  __syncthreads();
  if (s_flag[0] != 0 && warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES && s < nk; ++s) {
      // Phase parity of the last arming of stage s.
      const int uses = (nk - s + STAGES - 1) / STAGES;
      if (!mbar_wait(&full[s], (uses - 1) & 1)) report_status(p.status, PI05_DEV_TIMEOUT_DRAIN);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_acc, kTmemCols);
  }
}

template <int EPI, int TOK, int STAGES>
int launch_one(const SkinnyParams& p, const CUtensorMap& w0, const CUtensorMap& w1, const CUtensorMap& x,
               int tok_tiles, cudaStream_t stream) {
  constexpr int kSmemMax = smem_bytes<TOK, STAGES>();
  // Without a folded norm its area is left out.
  const int kSmem = p.fold_ssq != nullptr ? kSmemMax : smem_base_bytes<TOK, STAGES>();
  auto kern = skinny_gemm_kernel<EPI, TOK, STAGES>;
  static bool attr_done[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
    if (e != cudaSuccess) {
      set_last_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      return PI05_ERR_LAUNCH;
    }
    attr_done[dev] = true;
  }
  if (!p.cluster)
    return launch_pdl(kern, dim3(p.n_tiles * p.splits, tok_tiles), dim3(kThreads), kSmem, stream, pdl_enabled(),
                      w0, w1, x, p);
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(p.n_tiles * p.splits, tok_tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, w0, w1, x, p);
  count_launch();
  if (e != cudaSuccess) {
    set_last_error("cluster launch failed (splits %d): %s", p.splits, cudaGetErrorString(e));
    return PI05_ERR_LAUNCH;
  }
  return PI05_OK;
}

// Largest cluster size usable for this kernel instantiation on the current device
// (queried once per device: clusters of `s` CTAs with this kernel's resources).
template <int EPI, int TOK, int STAGES>
int max_cluster_size() {
  constexpr int kSmem = smem_base_bytes<TOK, STAGES>();
  static int cached[16] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && cached[dev]) return cached[dev];
  auto kern = skinny_gemm_kernel<EPI, TOK, STAGES>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes<TOK, STAGES>());
  cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  int best = 1;
  for (int s = 2; s <= 16; ++s) {
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(s * 8, 1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = s;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) best = s;
    else cudaGetLastError();
  }
  if (dev < 16) cached[dev] = best;
  return best;
}

int num_sms() {
  static int cached[16] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && cached[dev]) return cached[dev];
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 16) cached[dev] = n;
  return n;
}

}  // namespace

int row_ssq_parts(int m_tok, int n_cols) {
  return (m_tok >= kWideMinTokens && !wide_disabled()) ? n_cols / 64 : n_cols / 128;
}

int skinny_choose_splits(int n_tiles, int kb_total, int tok_tiles, int sms) {
  // Minimise (waves x k-blocks per CTA) plus a small per-split reduction cost.
  int best = 1;
  double best_cost = 1e30;
  const int max_s = std::min(kb_total, 32);
  for (int s = 1; s <= max_s; ++s) {
    const long units = (long)n_tiles * s * tok_tiles;
    if (s > 1 && units > sms) break;  // split grids must fit in one wave (tile barrier)
    const long waves = (units + sms - 1) / sms;
    const int kb_per = (kb_total + s - 1) / s;
    const double cost = (double)waves * (kb_per + 1.5) + (s > 1 ? 0.75 : 0.0);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

int skinny_choose_splits_cluster(int n_tiles, int kb_total, int tok_tiles, int sms, int max_cluster) {
  // Splits reduce inside a cluster, so any number of waves is legal; minimise
  // (waves x k-blocks per CTA) with a small cost per extra split.
  int best = 1;
  double best_cost = 1e30;
  const int max_s = std::min(kb_total, max_cluster);
  for (int s = 1; s <= max_s; ++s) {
    const long units = (long)n_tiles * s * tok_tiles;
    const long waves = (units + sms - 1) / sms;
    const int kb_per = (kb_total + s - 1) / s;
    const double cost = (double)waves * (kb_per + 1.5) + 0.15 * (s - 1);
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

int skinny_gemm_run(int epi, SkinnyParams p, const void* w0, const void* w1, int w_rows0, int w_rows1,
                    const void* x, int ldx, int splits_override, void* stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.m_tok <= 0 || p.k <= 0 || p.k % 8 != 0 || p.n_tiles <= 0 || (p.n_valid % 8) != 0) {
    set_last_error("skinny_gemm: bad shape m=%d k=%d tiles=%d", p.m_tok, p.k, p.n_tiles);
    return PI05_ERR_SHAPE;
  }
  const bool wide_ok = p.m_tok >= kWideMinTokens && p.allow_wide != 0 && !wide_disabled();
  if (p.fold_ssq != nullptr && epi == SK_EPI_STORE) {
    // Folded LayerNorm: many-token kernel only, sums, sums of squares and column sums.
    if (!wide_ok || p.ln_sum == nullptr || p.ln_colsum == nullptr || p.fold_parts <= 0 || p.fold_d <= 0 ||
        p.fold_ld < p.m_tok || p.fold_bias0 != nullptr || p.fold_bias1 != nullptr) {
      set_last_error("skinny_gemm: folded LayerNorm needs >= %d tokens, row sums, sums of squares and column sums",
                     kWideMinTokens);
      return PI05_ERR_SHAPE;
    }
  } else if (p.fold_ssq != nullptr) {
    // Small-token kernel: <= 64 tokens, rstd and the folded bias (denoise adaRMS);
    // many-token kernel: rstd only (the prefix LM's RMSNorm has no shift).
    bool bad = (epi != SK_EPI_GEGLU && epi != SK_EPI_QKV_ROPE) || p.fold_parts <= 0 || p.fold_d <= 0 ||
               p.fold_ld < p.m_tok || p.ln_sum != nullptr;
    if (wide_ok)
      bad = bad || p.fold_bias0 != nullptr || p.fold_bias1 != nullptr ||
            (epi == SK_EPI_QKV_ROPE && p.head_dim != 256);
    else
      bad = bad || (p.m_tok > 64 && p.max_tok != 64) || p.fold_parts > kNormMaxParts || p.fold_bias0 == nullptr ||
            p.fold_bias1 == nullptr;
    if (bad) {
      set_last_error("skinny_gemm: folded norm needs gate/up or q|k|v; 64-token tiles with 1..%d parts and both bias "
                     "vectors, or >= %d tokens without bias", kNormMaxParts, kWideMinTokens);
      return PI05_ERR_SHAPE;
    }
  }
  if (wide_ok) {
    int n_cols = 0;
    if (epi == SK_EPI_GEGLU)
      n_cols = p.n_tiles * 64;
    else if (epi == SK_EPI_QKV_ROPE)
      n_cols = (p.n_q_heads + 2 * p.n_kv_heads) * p.head_dim;
    else
      n_cols = p.n_valid > 0 ? p.n_valid : p.n_tiles * kBM;
    if (epi != SK_EPI_QKV_ROPE || p.head_dim == 256)
      return wide_gemm_run(epi, p, w0, w1, w_rows0, w_rows1, n_cols, x, ldx, stream);
  }
  const int tok = (p.m_tok <= 64 || p.max_tok == 64) ? 64 : (p.m_tok <= 128 ? 128 : 256);
  const int tok_tiles = (p.m_tok + tok - 1) / tok;
  p.kb_total = (p.k + kBK - 1) / kBK;
  int max_cl = 1;
  {
    constexpr int S = 4;
    switch (epi) {
#define PI05_SK_MAXCL(E)                                                      \
  case E:                                                                     \
    max_cl = tok == 64    ? max_cluster_size<E, 64, 3>()                      \
             : tok == 128 ? max_cluster_size<E, 128, S>()                     \
                          : max_cluster_size<E, 256, 3>();                    \
    break;
      PI05_SK_MAXCL(SK_EPI_STORE)
      PI05_SK_MAXCL(SK_EPI_GATED_RESID)
      PI05_SK_MAXCL(SK_EPI_GEGLU)
      PI05_SK_MAXCL(SK_EPI_QKV_ROPE)
#undef PI05_SK_MAXCL
      default:
        break;
    }
  }
  // An armed failure hook (pi05_debug_set_fault) selects the global split-K path it acts on.
  const DebugFault fault = debug_fault();
  if (fault.skip_split >= 0) {
    p.fault_skip_split = fault.skip_split;
    p.wait_ns = fault.wait_ns;
  }
  const bool use_cluster = p.allow_cluster != 0 && max_cl > 1 && fault.skip_split < 0;
  if (splits_override > 0) {
    p.splits = std::min(splits_override, p.kb_total);
    p.cluster = (use_cluster && p.splits > 1 && p.splits <= max_cl) ? 1 : 0;
  } else if (use_cluster) {
    // Small-token CTAs other than QKV+RoPE fit two per SM.
    const int slots = num_sms() * ((tok <= 128 && epi != SK_EPI_QKV_ROPE) ? 2 : 1);
    p.splits = skinny_choose_splits_cluster(p.n_tiles, p.kb_total, tok_tiles, slots, max_cl);
    p.cluster = p.splits > 1 ? 1 : 0;
  } else {
    p.splits = skinny_choose_splits(p.n_tiles, p.kb_total, tok_tiles, num_sms());
    p.cluster = 0;
  }
  if (p.splits > 1 && !p.cluster) {
    const size_t need = (size_t)tok_tiles * p.n_tiles * p.splits * tok * kBM * sizeof(float);
    if ((long)tok_tiles * p.n_tiles * p.splits > num_sms()) {
      set_last_error("skinny_gemm: split grid (%d CTAs) exceeds one wave", tok_tiles * p.n_tiles * p.splits);
      return PI05_ERR_SHAPE;
    }
    if (p.accum == nullptr || p.counters == nullptr || need > p.accum_bytes ||
        2 * tok_tiles * p.n_tiles > kWsNormTicketBase) {
      set_last_error("skinny_gemm: workspace too small (%zu needed)", need);
      return PI05_ERR_WORKSPACE;
    }
  }
  // Push-form split-K for the small-token tile (splits <= 16 fit its receive slots).
  {
    const int mt = std::min(p.m_tok, tok);
    const long need = (long)(p.splits - 1) * ((mt + p.splits - 1) / p.splits) * kBM * 4;
    p.push = (p.cluster && tok == 64 && p.splits <= 16 && need <= 32768) ? 1 : 0;
  }
  CUtensorMap tw0, tw1, tx;
  int rc = make_tmap_bf16_2d(&tw0, w0, w_rows0, p.k, p.k, 64, 64, true);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tw1, w1, w_rows1, p.k, p.k, 64, 64, true);
  if (rc) return rc;
  rc = make_tmap_bf16_2d(&tx, x, p.m_tok, p.k, ldx, tok, 64, true);
  if (rc) return rc;
  constexpr int S = 4;
  switch (epi) {
#define PI05_SK_CASE(E)                                                                 \
  case E:                                                                               \
    if (tok == 64)                                                                      \
      rc = launch_one<E, 64, 3>(p, tw0, tw1, tx, tok_tiles, st);                        \
    else if (tok == 128)                                                                \
      rc = launch_one<E, 128, S>(p, tw0, tw1, tx, tok_tiles, st);                       \
    else                                                                                \
      rc = launch_one<E, 256, 3>(p, tw0, tw1, tx, tok_tiles, st);                       \
    break;
    PI05_SK_CASE(SK_EPI_STORE)
    PI05_SK_CASE(SK_EPI_GATED_RESID)
    PI05_SK_CASE(SK_EPI_GEGLU)
    PI05_SK_CASE(SK_EPI_QKV_ROPE)
#undef PI05_SK_CASE
    default:
      set_last_error("skinny_gemm: unknown epilogue %d", epi);
      return PI05_ERR_INVALID_ARG;
  }
  return rc;
}

}  // namespace pi05
