// Tensor-core (tcgen05 / TMEM) skinny GEMM for 9..128 token rows: batched
// decode and speculative verify.  See gemm_tc.cu for the design.
#pragma once
#include "gemv.cuh"

namespace sb {

// Formats with a tensor-core tile copy of the weight (SbLinear.w_tc).
__host__ __device__ inline bool tc_format(int fmt) { return fmt == SB_FMT_FP8 || fmt == SB_FMT_BF16; }

// Geometry of one launch.
struct TcPlan {
  int mp;      // token rows padded (multiple of 8 for fp8, 16 for bf16)
  int np;      // MMA N = B-operand rows: 2*mp (fp8: two e4m3 terms) or mp (bf16)
  int tiles;   // 128-row weight tiles
  int kb;      // 128-byte K blocks
  int split;   // CTAs per cluster splitting K (1 = persistent over tiles)
  int stages;  // ring depth
  int ncols;   // TMEM columns allocated
  int n_ctas;
  size_t smem;
};

// Shared-memory layout, computed identically on the host and in the kernel.
struct TcLayout {
  size_t stage_bytes, part, out, bars, tmem, flag, best, bval, shift, total;
};
__host__ __device__ inline TcLayout tc_layout(int np, int stages, int m, int split) {
  auto up = [](size_t x, size_t a) { return (x + a - 1) & ~(a - 1); };
  TcLayout L;
  L.stage_bytes = 16384 + static_cast<size_t>(np) * 128;
  L.part = L.stage_bytes * stages;
  const size_t part_bytes = static_cast<size_t>(128) * m * 4;
  L.out = up(L.part + part_bytes, 16);
  const int rows_out = split > 1 ? (128 + split - 1) / split : 0;
  L.bars = up(L.out + static_cast<size_t>(rows_out) * m * 4, 16);
  L.tmem = up(L.bars + 8 * static_cast<size_t>(2 * stages + 2), 16);
  L.flag = L.tmem + 16;
  L.best = L.flag + 16;
  L.bval = L.best + 128 * 4;
  L.shift = L.bval + 128 * 4;
  L.total = L.shift + 128 * 4;
  return L;
}

// Bytes of the prepared B operand (activation terms) plus the per-row shifts.
size_t tc_operand_bytes(int fmt, int k, int m);
bool tc_plan(int fmt, int n, int k, int m, TcPlan& pl);
// p: the GEMV parameters (prologue + epilogue); w_tc: tile copy of the weight;
// operand: tc_operand_bytes() of scratch (device).
int tc_launch(const GemvParams& p, const void* w_tc, void* operand, const TcPlan& pl, int fmt, bool pdl,
              cudaStream_t stream);

}  // namespace sb
