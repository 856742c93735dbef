// Tensor-core (tcgen05 / TMEM) skinny GEMM for 9..128 token rows: batched
// decode and speculative verify.  See gemm_tc.cu for the design.
#pragma once
#include "gemv.cuh"

namespace sb {

// Every format can carry a tensor-core tile copy of the weight (SbLinear.w_tc):
// FP8 as its e4m3 bytes (the activations then enter as two e4m3 terms), the
// others as bf16 values (bf16 weights; INT8 codes; NVFP4 code x block scale,
// all exact in bf16), their fp32 row / tensor scale applied in the epilogue.
__host__ __device__ inline bool tc_format(int fmt) { return fmt >= SB_FMT_BF16 && fmt <= SB_FMT_NVFP4; }
__host__ __device__ constexpr bool tc_bf16_operand(int fmt) { return fmt != SB_FMT_FP8; }

// Geometry of one launch.
struct TcPlan {
  int mp;      // token rows padded (multiple of 8 for fp8, 16 for bf16)
  int np;      // MMA N = B-operand rows: 2*mp (fp8: two e4m3 terms) or mp (bf16)
  int tiles;   // 128-row weight tiles
  int kb;      // 128-byte K blocks
  int mtiles;  // token tiles of mp rows (> 1 only for the store epilogue: prefill)
  int split;   // CTAs per cluster splitting K (1 = persistent over tiles)
  int stages;  // ring depth
  int ncols;   // TMEM columns of the two accumulators (allocated, unless bs)
  int bs;      // block-scaled operand: TMEM also holds the scales (tmem_cols allocated)
  int tmem_cols;
  int epi_warps;  // epilogue warps (the block has epi_warps + 2)
  int n_ctas;
  size_t smem;
};

// Shared-memory layout, computed identically on the host and in the kernel.
struct TcLayout {
  size_t stage_bytes, part, out, bars, tmem, flag, best, bval, shift, wbv, wbi, live, sfa, total;
};
__host__ __device__ inline int tc_rows_per_rank(int split) {
  const int rp = (128 + split - 1) / split;
  return (rp + 1) & ~1;  // even: RoPE / gate-up row pairs stay in one CTA
}
// floats per inbox row: whole 8-token chunks (16-byte aligned stores) + 4 (bank spread)
__host__ __device__ inline int tc_inbox_stride(int m) { return (m + 7) / 8 * 8 + 4; }
// warps of a tcgen05 GEMM block: epilogue warps (a multiple of 4: each TMEM
// lane quarter is read by epilogue_warps / 4 warps), producer, MMA.  The
// block-scaled GEMM (gemm_bs.cu) runs 8; this GEMM 16 with one CTA per SM and
// 8 with two (its register budget is the same for both).
constexpr int kTcEpiWarps = 8;
constexpr int kTcThreads = (kTcEpiWarps + 2) * 32;
constexpr int kTcMaxEpiWarps = 16;
// bs: the B operand carries block scales (512 bytes per stage) and the
// weight's unit scales take 512 bytes (tcgen05.mma kind::mxf8f6f4)
__host__ __device__ inline TcLayout tc_layout(int np, int stages, int m, int split, int epi_warps, bool bs = false) {
  auto up = [](size_t x, size_t a) { return (x + a - 1) & ~(a - 1); };
  TcLayout L;
  L.stage_bytes = 16384 + static_cast<size_t>(np) * 128 + (bs ? 512 : 0);
  L.part = L.stage_bytes * stages;
  // split > 1: inbox [split source ranks][rows per rank][tc_inbox_stride(m)] of K partials
  const size_t part_bytes =
      split > 1 ? static_cast<size_t>(split) * tc_rows_per_rank(split) * tc_inbox_stride(m) * 4 : 0;
  L.out = up(L.part + part_bytes, 16);
  L.bars = L.out;
  L.tmem = up(L.bars + 8 * static_cast<size_t>(2 * stages + 4), 16);
  L.flag = L.tmem + 16;
  L.best = L.flag + 16;
  L.bval = L.best + 128 * 4;
  L.shift = L.bval + 128 * 4;
  L.wbv = L.shift + 128 * 4;                    // [warps][128] running argmax value
  L.wbi = L.wbv + static_cast<size_t>(epi_warps + 2) * 128 * 4;   // [warps][128] running argmax index
  L.live = L.wbi + static_cast<size_t>(epi_warps + 2) * 128 * 4;  // [1 + 64] token tiles holding a real row (prefill)
  L.sfa = up(L.live + 65 * 4, 128);  // bs: 512 bytes of UE8M0 1.0 (the weight's block scales)
  L.total = bs ? L.sfa + 512 : L.live + 65 * 4;
  return L;
}

// Bytes of the prepared B operand (activation terms) plus the per-row shifts.
size_t tc_operand_bytes(int fmt, int k, int m);
bool tc_plan(int fmt, int n, int k, int m, TcPlan& pl);
// p: the GEMV parameters (prologue + epilogue); w_tc: tile copy of the weight;
// operand: tc_operand_bytes() of scratch (device).  operand_ready: the
// preceding kernel has written the operand (one token tile) and, for fp8, one
// row of shifts per K-split rank (rank r's K range scaled by 2^xshift[r][m]),
// so no preparation kernel runs.
int tc_launch(const GemvParams& p, const void* w_tc, void* operand, const TcPlan& pl, int fmt, bool pdl,
              cudaStream_t stream, bool operand_ready = false);
// where the shifts start inside an operand of tc_operand_bytes(fmt, k, m)
size_t tc_shift_offset(int fmt, int k, int m);

// Tensor-core decode chain (fp8 weights, 9..64 token rows, one token tile):
// the GEMM reads a block-scaled operand that the preceding GEMM's epilogue
// wrote (operand.cuh) instead of a prepared one.  max_split: the widest K
// split the plan may use (1 for a SwiGLU producer, whose 32-element blocks
// span two warps of one CTA).
bool tc_plan_bs(int n, int k, int m, int max_split, TcPlan& pl);
size_t tc_bs_operand_bytes(int k, int m);
int tc_launch_bs(const GemvParams& p, const void* w_tc, const void* operand, const TcPlan& pl, bool pdl,
                 cudaStream_t stream);

}  // namespace sb
