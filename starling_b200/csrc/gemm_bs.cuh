// NVFP4 block-scaled tensor-core GEMV/GEMM for 1..8 token rows (B = 1 decode,
// speculative verify): tcgen05.mma kind::mxf4nvf4 with the weight's own e2m1
// codes and e4m3 block scales.  See gemm_bs.cu for the design.
#pragma once
#include "gemm_tc.cuh"

namespace sb {

constexpr int kBsTerms = 8;          // e2m1 terms per activation row (MMA N = 8 per token)
constexpr int kBsMaxRows = 8;        // token rows served: N = 8 * rows <= 64
constexpr int kBsCodeBytes = 16384;  // 128 rows x 256 e2m1 codes
constexpr int kBsBlock = 18432;      // one (128-row tile, 256-element K block) of SbLinear.w_bs: codes + scales

struct BsPlan {
  int m;          // token rows
  int ncol;       // MMA N = kBsTerms * m
  int tiles;      // 128-row weight tiles
  int kb;         // 256-element K blocks
  int kbc;        // K blocks of one cluster rank (at most)
  int split;      // CTAs per cluster splitting K (1 = persistent over tiles)
  int stages;     // ring depth
  int tmem_cols;  // TMEM columns allocated
  int sf_col;     // first TMEM column of the scale factors (A: 16 per stage, then B: 16 per K block)
  int n_ctas;
  size_t smem;
};

// Shared-memory layout, computed identically on the host and in the kernel.
struct BsLayout {
  size_t bops, sfb, bars, tmem, flag, gexp, rstd, amax, red, best, bval, wbv, wbi, part, total;
};
__host__ __device__ inline BsLayout bs_layout(int ncol, int kbc, int stages, int m, int split) {
  auto up = [](size_t x, size_t a) { return (x + a - 1) & ~(a - 1); };
  BsLayout L;
  L.bops = static_cast<size_t>(stages) * kBsBlock;                    // ring of weight blocks first
  L.sfb = L.bops + static_cast<size_t>(kbc) * ncol * 128;              // B codes, resident
  L.bars = L.sfb + static_cast<size_t>(kbc) * 2048;                    // B scales, resident
  L.tmem = up(L.bars + 8 * static_cast<size_t>(2 * stages + 5), 16);  // full, empty, acc[2][2], B ready
  L.flag = L.tmem + 16;
  L.gexp = L.flag + 16;  // [8] per-token exponent of the term scales
  L.rstd = L.gexp + 32;  // [8] RMSNorm 1/rms
  L.amax = L.rstd + 32;  // [8] max |activation| (float bits)
  L.red = L.amax + 32;   // [2][8 warps][8 tokens]
  L.best = L.red + 512;
  L.bval = L.best + 32;
  L.wbv = L.bval + 32;                                   // [warps][128] running argmax value
  L.wbi = L.wbv + (kTcEpiWarps + 2) * 128 * 4;           // [warps][128] running argmax index
  L.part = up(L.wbi + (kTcEpiWarps + 2) * 128 * 4, 16);  // split > 1: inbox of K partials
  L.total = L.part + (split > 1 ? static_cast<size_t>(split) * tc_rows_per_rank(split) * tc_inbox_stride(m) * 4 : 0);
  return L;
}

bool bs_plan(int n, int k, int m, BsPlan& pl);
// p: GEMV parameters (prologue + epilogue, p.m token rows); w_bs: SbLinear.w_bs.
int bs_launch(const GemvParams& p, const void* w_bs, const BsPlan& pl, bool pdl, cudaStream_t stream);

}  // namespace sb
