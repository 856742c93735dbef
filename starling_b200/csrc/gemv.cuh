// Dequant-GEMV ("skinny GEMM", m <= 64 token rows) with fused prologue and
// epilogue.  See gemv.cu for the kernel and the design notes.
#pragma once
#include "common.cuh"

namespace sb {

enum { PRO_NONE = 0, PRO_RMSNORM = 1, PRO_EMBED = 2 };
enum { EPI_STORE = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_ARGMAX = 4 };

struct GemvParams {
  // packed weight
  const uint8_t* w;
  const uint8_t* scale;
  float gscale;
  int n;         // logical rows
  int k;
  int n_tiles;   // n_pad / 16
  int kg_total;  // k / kgroup elements
  // launch configuration
  int rt;  // row tiles per CTA (cluster)
  int ck;  // CTAs per cluster splitting K
  int m;   // token rows (<= 64)
  // prologue
  int pro;
  const uint16_t* x;       // [m][k] input rows (PRO_NONE / PRO_RMSNORM)
  const uint16_t* norm_w;  // [k] RMSNorm weight
  float eps;
  const int64_t* ids;      // PRO_EMBED: token id per row
  const uint16_t* embed;   // PRO_EMBED: [vocab][k]
  int embed_rows;          // PRO_EMBED: vocab (ids are clamped into range)
  float emb_mult;
  uint16_t* hidden_out;    // PRO_EMBED: the embedded rows are written here
  // epilogue
  int epi;
  uint16_t* y;  // STORE [m][n]; RESID hidden [m][n] (in place); SWIGLU act [m][n/2]
  float res_mult;
  // EPI_QKV
  uint16_t* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
  int n_q, n_kv, max_len, m_per;  // m_per = tokens per stream
  const uint16_t* cos_tab;
  const uint16_t* sin_tab;
  int rope_max;
  const int32_t* rope_off;
  int32_t* ctrl;
  // EPI_ARGMAX
  uint16_t* logits;
  float logits_mult;
  float* part_val;
  int* part_idx;
  int* counter;
  int n_ctas;  // CTAs that produce argmax partials (= grid when ck == 1)
  int mode;
  int batch;
  int step;
  int64_t* ids_io;
  int64_t* out_ids;
  int32_t* finished;
  int64_t eos_id;
  int64_t pad_id;
  // optional shared-memory copies (fused step, step.cu); null elsewhere
  const uint16_t* rope_cache;  // EPI_QKV: [m][cos 64 | sin 64] at each token's position
  uint16_t* resid_cache;       // EPI_RESID: [m][rc_stride] rows rc_row0.. of y, kept in step with y
  int rc_stride, rc_row0;
  // prefill of right-padded prompts (tensor-core GEMM): token m is stream
  // row_b0 + m / row_T at position m % row_T, padding when that position is
  // >= row_len[stream]; null: no padding
  const int32_t* row_len;
  int row_T, row_b0;
  // tensor-core decode chain (gemm_tc.cu), null elsewhere.  Producer (EPI_RESID,
  // EPI_SWIGLU): the epilogue also writes the next projection's block-scaled
  // fp8 operand nx_op (np = nx_np rows, token m's terms in rows m and nx_mp + m)
  // of its new rows times nx_g (the next RMSNorm weight; null: none) and, for
  // EPI_RESID, nx_ssq[m * (n / 32) + j] = the sum of squares of token m's new
  // rows 32 j .. 32 j + 31.  Consumer: ssq_in (the producer's nx_ssq) gives
  // each token's RMSNorm 1 / rms, applied to its outputs; null: none.
  uint8_t* nx_op;
  const uint16_t* nx_g;
  float* nx_ssq;
  int nx_np, nx_mp;
  const float* ssq_in;
};

template <int FMT>
struct KG {
  static constexpr int E = FMT == SB_FMT_NVFP4 ? 64 : (FMT == SB_FMT_BF16 ? 16 : 32);  // K elements per kgroup
  static constexpr int KS = E / 16;                                                  // mma k-steps per kgroup
};

// launch plan of the persistent decode GEMV (gemv_dec.cu)
struct DecPlan {
  int ksw, warps, slots, batch, n_ctas;
  size_t smem;
};
// Shared-memory layout of the decode GEMV, computed identically on the host
// (allocation size) and in the kernel (offsets).  All offsets 16-aligned.
struct DecLayout {
  size_t slot_bytes, bars, red, tot, ss, shift, best, bval, flag, xs, total;
};
__host__ __device__ inline DecLayout dec_layout(size_t tile_bytes, int slots, int batch, int warps, int m, int kw) {
  auto up16 = [](size_t x) { return (x + 15) & ~size_t(15); };
  DecLayout L;
  L.slot_bytes = (tile_bytes + 127) & ~size_t(127);
  L.bars = L.slot_bytes * slots;
  L.red = up16(L.bars + 8 * static_cast<size_t>(slots));
  L.tot = up16(L.red + static_cast<size_t>(batch) * warps * 16 * m * 4);
  L.ss = up16(L.tot + static_cast<size_t>(batch) * 16 * m * 4);
  L.shift = up16(L.ss + 128 * 4);
  L.best = up16(L.shift + 128 * 4);
  L.bval = up16(L.best + 8 * 4);
  L.flag = up16(L.bval + 8 * 4);
  L.xs = up16(L.flag + 16);  // [warps][m][kw + 8] activation slices
  L.total = up16(L.xs + static_cast<size_t>(warps) * m * (kw + 8) * 2);
  return L;
}
bool gemv_dec_plan(int fmt, int n_tiles, int k, int m, DecPlan& pl);
int gemv_dec_launch(const GemvParams& p, const DecPlan& pl, int fmt, bool pdl, cudaStream_t stream);

struct GemvCfg {
  int rt, ck, warps, nt;
};

int kgroup_elems(int fmt);
GemvCfg gemv_pick(int fmt, int n_pad, int k, int m);
size_t gemv_smem_bytes(const GemvCfg& c, int k, int m);
int gemv_grid(const GemvCfg& c, int n_tiles);
int gemv_launch(const GemvParams& p, const GemvCfg& c, int fmt, bool pdl, cudaStream_t stream);

}  // namespace sb
