// Persistent tcgen05 GEMM for many-token projections (tokens as UMMA M).
#pragma once

#include "skinny_gemm.h"

namespace pi05 {

// Same parameter block and epilogue kinds as the small-token kernel.  n_cols:
// output columns (GEGLU: intermediate width; QKV_ROPE: (n_q + 2 n_kv) * 256).
int wide_gemm_run(int epi, SkinnyParams p, const void* w0, const void* w1, int w_rows0, int w_rows1, int n_cols,
                  const void* x, int ldx, void* stream);

// Tile width (128 / 192 / 256), split-K count and the CTA grouping for an epilogue
// kind and shape: *pair = 0 single CTAs, 1 a CTA pair shares each tile (cta_group::2,
// 256 x 256 tiles), 2 cluster split-K (two CTAs take the K halves of a 128-column
// tile and exchange partials SM to SM); m_tiles counts 128-token tiles.
int wide_choose(int epi, int m_tiles, int n_cols, int kb_total, int sms, int* bn, int* splits, int* pair,
                bool allow_pair = true);

// PI05_WIDE=0 in the environment keeps every projection on the small-token kernel.
bool wide_disabled();

// Token count above which skinny_gemm_run hands a projection to the wide kernel.
constexpr int kWideMinTokens = 129;

}  // namespace pi05
