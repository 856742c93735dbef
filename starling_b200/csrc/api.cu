// C ABI of libstarling_b200 (declared in include/starling_b200.h) and the
// host-side sequencing of one decode / verify forward.
//
// sb_decode_step issues, per layer, five launches on the caller's stream:
//   1. q/k/v dequant-GEMV   RMSNorm prologue (layer 0: embedding x12 + RMSNorm),
//                           RoPE + KV-cache write epilogue
//   2. attention            cluster split over the context
//   3. o dequant-GEMV       residual epilogue into the hidden rows
//   4. gate/up GEMV         RMSNorm prologue, SiLU*up epilogue
//   5. down GEMV            residual epilogue
// and finally the lm_head GEMV with the final RMSNorm prologue and the fused
// argmax / token feedback epilogue.  Every dynamic value (token ids, cache
// slot, finished flags) is read from device memory, so the launches can be
// captured once into a CUDA graph and replayed.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "attention.cuh"
#include "gemm_bs.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "glue.cuh"
#include "step.cuh"

#include <atomic>

using namespace sb;

static thread_local char g_err[1024] = "";
static std::atomic<unsigned long long> g_launches{0};
void sb::note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
int sb::set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

#define SB_TRY(expr)                                                                                   \
  do {                                                                                                 \
    int _rc = (expr);                                                                                  \
    if (_rc != 0) {                                                                                    \
      if (_rc < 1000) return fail(_rc, "%s: %s", #expr, cudaGetErrorString(static_cast<cudaError_t>(_rc))); \
      return _rc;                                                                                      \
    }                                                                                                  \
  } while (0)

static bool lin_ok(const SbLinear& l) {
  if (!l.w || l.n <= 0 || l.k <= 0 || l.n_pad < l.n || (l.n_pad % 16) != 0) return false;
  if (l.fmt < SB_FMT_BF16 || l.fmt > SB_FMT_NVFP4) return false;
  if (l.k % kgroup_elems(l.fmt) != 0 || l.k % 64 != 0) return false;
  if (l.fmt != SB_FMT_BF16 && !l.scale) return false;
  return true;
}

static GemvParams base_params(const SbLinear& l, int m) {
  GemvParams p;
  memset(&p, 0, sizeof(p));
  p.w = static_cast<const uint8_t*>(l.w);
  p.scale = static_cast<const uint8_t*>(l.scale);
  p.gscale = l.global_scale;
  p.n = l.n;
  p.k = l.k;
  p.n_tiles = l.n_pad / 16;
  p.kg_total = l.k / kgroup_elems(l.fmt);
  p.m = m;
  return p;
}

static bool dec_plan_for(int fmt, int n_tiles, int k, int m, DecPlan& pl) {
  return gemv_dec_plan(fmt, n_tiles, k, m, pl);
}

// The tcgen05 path serves a linear with a tile copy above 8 token rows (FP8,
// bf16: the copy has the packed weight's bytes) or above 64 rows (NVFP4, INT8:
// the bf16 copy has 4x / 2x the bytes, worth it only where the work is
// compute-bound, i.e. prefill).
static bool tc_plan_for(const SbLinear& l, int m, TcPlan& pl) {
  const int min_rows = (l.fmt == SB_FMT_NVFP4 || l.fmt == SB_FMT_INT8) ? 64 : 8;
  return m > min_rows && l.w_tc && tc_plan(l.fmt, l.n, l.k, m, pl);
}

// Tensor-core decode chain (fp8 weights, 9..64 token rows, every layer): the
// o and down GEMMs' residual epilogues and the gate/up GEMM's SwiGLU epilogue
// write the next projection's block-scaled operand -- with, after a residual,
// per-32-row sums of squares for the RMSNorm that follows -- so q/k/v (layers
// >= 1), gate/up and down run without a preparation launch.  Layer 0's q/k/v
// (embedding input) and the lm_head keep theirs.
struct ChainPlan {
  TcPlan qkv, gu, down;  // the consumers' block-scaled plans
};
static bool chain_plan(const SbModel* md, int T, ChainPlan& c) {
  if (!md->layers || md->n_layers < 1 || T < 9 || T > 64) return false;
  for (int l = 0; l < md->n_layers; ++l) {
    const SbLayer& L = md->layers[l];
    const SbLinear* lins[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
    for (const SbLinear* x : lins)
      if (x->fmt != SB_FMT_FP8 || !x->w_tc) return false;
  }
  const SbLayer& L = md->layers[0];
  TcPlan op;  // o keeps its own operand (the attention's) and only produces
  if (!tc_plan_for(L.o, T, op) || op.mtiles != 1 || (op.split != 2 && op.split != 4) || op.epi_warps != kTcMaxEpiWarps)
    return false;
  // a producer writes whole 32-element blocks from one CTA: a residual GEMM
  // the rows of its rank (K split 2 or 4: 64 or 32 rows), the SwiGLU GEMM a
  // whole tile's 64 activations (no K split)
  if (!tc_plan_bs(L.qkv.n, L.qkv.k, T, 8, c.qkv) || !tc_plan_bs(L.gate_up.n, L.gate_up.k, T, 1, c.gu) ||
      !tc_plan_bs(L.down.n, L.down.k, T, 4, c.down))
    return false;
  return c.gu.split == 1 && (c.down.split == 2 || c.down.split == 4) && L.o.n % 128 == 0 && L.down.k % 128 == 0 &&
         L.qkv.k == L.o.n && L.gate_up.k == L.o.n && L.gate_up.n == 2 * L.down.k;
}

static int run_gemv(GemvParams& p, int fmt, bool pdl, cudaStream_t s) {
  DecPlan pl;
  if (p.m <= 8 && dec_plan_for(fmt, p.n_tiles, p.k, p.m, pl)) {
    const int rc = gemv_dec_launch(p, pl, fmt, pdl, s);
    if (rc != 0) return fail(rc, "decode gemv launch (n=%d k=%d m=%d): %s", p.n, p.k, p.m,
                             rc < 1000 ? cudaGetErrorString((cudaError_t)rc) : "config");
    return 0;
  }
  const GemvCfg c = gemv_pick(fmt, p.n_tiles * 16, p.k, p.m < 64 ? p.m : 64);
  p.rt = c.rt;
  p.ck = c.ck;
  if (p.k % (c.ck * kgroup_elems(fmt)) != 0) return fail(SB_ERR_CONFIG, "k=%d not divisible for ck=%d", p.k, c.ck);
  const int rc = gemv_launch(p, c, fmt, pdl, s);
  if (rc == SB_ERR_CONFIG)
    return fail(rc, "no gemv configuration for n=%d k=%d m=%d (smem %zu)", p.n, p.k, p.m, gemv_smem_bytes(c, p.k, p.m < 64 ? p.m : 64));
  if (rc != 0) return fail(rc, "gemv launch (n=%d k=%d m=%d): %s", p.n, p.k, p.m, cudaGetErrorString((cudaError_t)rc));
  return 0;
}

// NVFP4 1..8-row path (sb_set_nvfp4_path)
static std::atomic<int> g_nvfp4_path{SB_NVFP4_AUTO};
static int nvfp4_path() { return g_nvfp4_path.load(std::memory_order_relaxed); }

// Whether the block-scaled kernel serves (l, m).  In auto mode it takes the
// shapes where it measured faster than the mma.sync GEMV on B200 (graphed
// launches, weights streamed from HBM): its fixed cost per launch (TMEM
// allocation, building the activation terms, ~100 ns per tcgen05 instruction)
// is paid back over hundreds of tiles (lm_head: 24.7 vs 42.5 us at 1 row,
// 52 vs 131 us at 8) and by every 8-row forward (q/k/v 9.0 vs 10.8, o 8.5 vs
// 9.7, gate/up 18.9 vs 25.2, down 18.5 vs 22.6 us), not by the 1-row layer
// projections (gate/up 9.7 vs 9.3, q/k/v 7.3 vs 4.3 us).
static bool bs_serves(const SbLinear& l, int m, BsPlan& bp) {
  if (l.fmt != SB_FMT_NVFP4 || !l.w_bs || m > kBsMaxRows) return false;
  const int mode = nvfp4_path();
  if (mode == SB_NVFP4_MMA_SYNC || !bs_plan(l.n, l.k, m, bp)) return false;
  if (mode == SB_NVFP4_BLOCK_SCALED) return true;
  return bp.tiles >= 256 || m >= 8;
}

int32_t sb_set_nvfp4_path(int32_t mode) {
  if (mode < SB_NVFP4_AUTO || mode > SB_NVFP4_MMA_SYNC) return fail(SB_ERR_ARG, "sb_set_nvfp4_path: mode %d", mode);
  const int prev = nvfp4_path();
  g_nvfp4_path.store(mode, std::memory_order_relaxed);
  return prev;
}

// 1..8 token rows: the block-scaled tcgen05 kernel where bs_serves, else the
// GEMV kernels.
static int run_small(const SbLinear& l, GemvParams& p, bool pdl, cudaStream_t s) {
  BsPlan bp;
  if (bs_serves(l, p.m, bp)) {
    const int rc = bs_launch(p, l.w_bs, bp, pdl, s);
    if (rc != 0) return fail(rc, "block-scaled gemm launch (n=%d k=%d m=%d): %s", p.n, p.k, p.m,
                             rc < 1000 ? cudaGetErrorString((cudaError_t)rc) : "config");
    return 0;
  }
  return run_gemv(p, l.fmt, pdl, s);
}

// One linear: the tcgen05 GEMM when it serves (l, p.m) and operand scratch is
// given, else run_small.
static int run_linear(const SbLinear& l, GemvParams& p, void* tc_scratch, size_t tc_bytes, bool pdl, cudaStream_t s) {
  TcPlan pl;
  if (tc_scratch && tc_plan_for(l, p.m, pl)) {
    const size_t need = tc_operand_bytes(l.fmt, l.k, p.m);
    if (need > tc_bytes) return fail(SB_ERR_ARG, "tensor-core operand scratch too small (%zu < %zu)", tc_bytes, need);
    const int rc = tc_launch(p, l.w_tc, tc_scratch, pl, l.fmt, pdl, s);
    if (rc != 0) return fail(rc, "tensor-core gemm launch (n=%d k=%d m=%d): %s", p.n, p.k, p.m,
                             rc < 1000 ? cudaGetErrorString((cudaError_t)rc) : "config");
    return 0;
  }
  return run_small(l, p, pdl, s);
}

// CTAs per (stream, KV head): enough (stream, head) groups fill the GPU on
// their own; few groups split their keys over a cluster of up to 8 CTAs.
static int attn_split(int groups, int max_len) {
  if (groups >= 148) return 1;
  int s = (2 * 148 + groups - 1) / groups;
  const int by_len = (max_len + 63) / 64;  // at least one 64-key tile per CTA
  if (s > by_len) s = by_len;
  return s < 1 ? 1 : (s > 8 ? 8 : s);
}

// need_workspace = false: the caller supplies the scratch itself
// (sb_lm_head_argmax_static), so state->workspace may be NULL.
static int check_state(const SbModel* md, const SbState* st, bool need_workspace = true) {
  if (!md || !st) return fail(SB_ERR_ARG, "null model/state");
  if (st->batch < 1 || st->m < 1 || st->batch * st->m > 64)
    return fail(SB_ERR_ARG, "batch*m must be in [1, 64] (batch=%d m=%d)", st->batch, st->m);
  if (st->batch > md->max_batch) return fail(SB_ERR_ARG, "batch %d > model max_batch %d", st->batch, md->max_batch);
  if (md->head_dim != 128) return fail(SB_ERR_ARG, "head_dim must be 128");
  if (md->n_q % md->n_kv != 0 || (md->n_q / md->n_kv) * st->m > 64)
    return fail(SB_ERR_ARG, "query rows per KV head (n_q/n_kv * m) must be <= 64");
  if (!st->ids || !st->ctrl || !st->hidden || !st->q || !st->attn || !st->act || (need_workspace && !st->workspace))
    return fail(SB_ERR_ARG, "state buffer missing");
  if (st->mode < SB_MODE_DECODE || st->mode > SB_MODE_FIRST) return fail(SB_ERR_ARG, "bad mode");
  return 0;
}

struct LmWork {
  float* val;
  int* idx;
  int* counter;
  int n_ctas;
  size_t bytes;
};

// exact = false: the partials are sized for the largest grid any kernel choice
// could use, so a workspace sized once stays valid when sb_set_nvfp4_path
// changes the choice later; exact = true: for the launch about to be issued
// only (scratch sized per call).
static LmWork lm_work(const SbModel* md, int tokens, void* base, bool exact = false) {
  const SbLinear& l = md->lm_head;
  LmWork w;
  DecPlan pl;
  TcPlan tp;
  BsPlan bp;
  const GemvCfg c = gemv_pick(l.fmt, l.n_pad, l.k, tokens);
  const int gemv_ctas = gemv_grid(c, l.n_pad / 16) / c.ck;
  const bool dec = tokens <= 8 && dec_plan_for(l.fmt, l.n_pad / 16, l.k, tokens, pl);
  const bool tc = tc_plan_for(l, tokens, tp);
  if (bs_serves(l, tokens, bp)) {
    w.n_ctas = bp.n_ctas;
  } else if (dec) {
    w.n_ctas = pl.n_ctas;
  } else if (tc) {
    w.n_ctas = tp.n_ctas;
  } else {
    w.n_ctas = gemv_ctas;
  }
  int n_max = gemv_ctas;
  if (dec && pl.n_ctas > n_max) n_max = pl.n_ctas;
  if (tc && tp.n_ctas > n_max) n_max = tp.n_ctas;
  BsPlan bq;
  if (l.fmt == SB_FMT_NVFP4 && l.w_bs && bs_plan(l.n, l.k, tokens, bq) && bq.n_ctas > n_max) n_max = bq.n_ctas;
  if (exact) n_max = w.n_ctas;
  if (w.n_ctas > n_max) n_max = w.n_ctas;
  const size_t pv = static_cast<size_t>(n_max) * tokens * 4;
  char* b = static_cast<char*>(base);
  w.counter = reinterpret_cast<int*>(b);
  w.val = reinterpret_cast<float*>(b + 256);
  w.idx = reinterpret_cast<int*>(b + 256 + ((pv + 255) & ~size_t(255)));
  w.bytes = 256 + 2 * ((pv + 255) & ~size_t(255));
  return w;
}

// Workspace = [lm_head argmax partials | tensor-core operand scratch | fused-step
// scratch | decode-chain operands: hidden-wide, inter-wide, sums of squares].
struct WsLayout {
  size_t lm_bytes, tc_off, tc_bytes, step_off, step_bytes, chain_off, chain_op1, chain_op2, chain_ssq, total;
  ChainPlan chain;  // valid when chain_off != 0
};
static size_t tc_scratch_need(const SbLinear& l, int tokens) {
  TcPlan pl;
  return tc_plan_for(l, tokens, pl) ? tc_operand_bytes(l.fmt, l.k, tokens) : 0;
}
static WsLayout ws_layout(const SbModel* md, int tokens) {
  WsLayout w{};
  w.lm_bytes = lm_work(md, tokens, nullptr).bytes;
  w.tc_off = (w.lm_bytes + 255) & ~size_t(255);
  size_t need = tc_scratch_need(md->lm_head, tokens);
  for (int l = 0; md->layers && l < md->n_layers; ++l) {
    const SbLayer& L = md->layers[l];
    const SbLinear* lins[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
    for (const SbLinear* x : lins) {
      const size_t b = tc_scratch_need(*x, tokens);
      if (b > need) need = b;
    }
  }
  w.tc_bytes = need;
  w.total = need ? w.tc_off + need : w.lm_bytes;
  w.step_bytes = md->n_q > 0 ? step_ws_bytes(md, tokens) : 0;
  w.step_off = (w.total + 255) & ~size_t(255);
  if (w.step_bytes) w.total = w.step_off + w.step_bytes;
  w.chain_off = w.chain_op1 = w.chain_op2 = w.chain_ssq = 0;
  if (chain_plan(md, tokens, w.chain)) {
    const SbLayer& L = md->layers[0];
    w.chain_off = (w.total + 255) & ~size_t(255);
    w.chain_op1 = (tc_bs_operand_bytes(L.o.n, tokens) + 255) & ~size_t(255);
    w.chain_op2 = (tc_bs_operand_bytes(L.down.k, tokens) + 255) & ~size_t(255);
    w.chain_ssq = static_cast<size_t>(L.o.n / 32) * 64 * 4;
    w.total = w.chain_off + w.chain_op1 + w.chain_op2 + w.chain_ssq;
  }
  return w;
}
// The state's workspace must hold ws_layout().total bytes; tc scratch is
// null when no linear of the model takes the tensor-core path at this size.
static int tc_scratch_of(const SbModel* md, const SbState* st, void*& ptr, size_t& bytes, WsLayout* out = nullptr) {
  const WsLayout w = ws_layout(md, st->batch * st->m);
  if (out) *out = w;
  if (st->workspace_bytes < w.total) return fail(SB_ERR_ARG, "workspace too small (%zu < %zu)", st->workspace_bytes, w.total);
  ptr = w.tc_bytes ? static_cast<char*>(st->workspace) + w.tc_off : nullptr;
  bytes = w.tc_bytes ? st->workspace_bytes - w.tc_off : 0;
  return 0;
}

// The decode chain's buffers inside the state's workspace (chain_plan holds).
struct ChainBufs {
  uint8_t* op1;  // hidden-wide operand: q/k/v's (from down) and gate/up's (from o)
  uint8_t* op2;  // inter-wide operand: down's (from gate/up)
  float* ssq;    // [64 tokens][hidden / 32] sums of squares of the last residual's rows
};
// (w: the state's ws_layout, its workspace already checked against w.total)
static void chain_bufs(const SbState* st, const WsLayout& w, ChainBufs& b) {
  char* base = static_cast<char*>(st->workspace) + w.chain_off;
  b.op1 = reinterpret_cast<uint8_t*>(base);
  b.op2 = reinterpret_cast<uint8_t*>(base + w.chain_op1);
  b.ssq = reinterpret_cast<float*>(base + w.chain_op1 + w.chain_op2);
}

// Token rows above which RMSNorm runs as its own kernel instead of the GEMV
// prologue (which every CTA of the GEMV would otherwise recompute).
static const int kFusedNormMaxRows = 8;

static int run_norm(const SbModel* md, const SbState* st, const uint16_t* x, bool embed, const uint16_t* w,
                    cudaStream_t s) {
  const int T = st->batch * st->m;
  if (!st->xnorm) return fail(SB_ERR_ARG, "state->xnorm is required for more than %d token rows", kFusedNormMaxRows);
  const int rc = norm_rows_launch(embed ? nullptr : x, embed ? st->ids : nullptr, md->embed, md->vocab, md->emb_mult, w,
                                  st->xnorm, embed ? st->hidden : nullptr, T, md->hidden, md->eps, st->use_pdl != 0, s);
  if (rc != 0) return fail(rc, "norm launch: %s", rc < 1000 ? cudaGetErrorString((cudaError_t)rc) : "config");
  return 0;
}

// Scratch of the lm_head launch alone: [argmax partials | 256-byte aligned
// tensor-core operand of the lm_head (only when the lm_head takes that path)].
struct LmLayout {
  size_t tc_off, tc_bytes, total;
};
static LmLayout lm_layout(const SbModel* md, int tokens) {
  LmLayout w;
  const size_t lm = lm_work(md, tokens, nullptr, true).bytes;
  w.tc_off = (lm + 255) & ~size_t(255);
  w.tc_bytes = tc_scratch_need(md->lm_head, tokens);
  w.total = w.tc_bytes ? w.tc_off + w.tc_bytes : lm;
  return w;
}

// lm_only: the state's workspace holds only lm_layout() (argmax partials,
// then the lm_head's own tensor-core operand) instead of the step's whole
// ws_layout().
static int launch_lm_head(const SbModel* md, const SbState* st, int step, cudaStream_t s, bool lm_only = false) {
  const int T = st->batch * st->m;
  LmWork w = lm_work(md, T, st->workspace, lm_only);
  if (w.bytes > st->workspace_bytes) return fail(SB_ERR_ARG, "workspace too small (%zu < %zu)", st->workspace_bytes, w.bytes);
  GemvParams p = base_params(md->lm_head, T);
  p.pro = PRO_RMSNORM;
  p.x = st->hidden;
  p.norm_w = md->final_norm;
  p.eps = md->eps;
  size_t tcb = 0;
  void* tcs = nullptr;
  if (lm_only) {
    const LmLayout lw = lm_layout(md, T);
    if (st->workspace_bytes < lw.total)
      return fail(SB_ERR_ARG, "workspace too small (%zu < %zu)", st->workspace_bytes, lw.total);
    tcs = lw.tc_bytes ? static_cast<char*>(st->workspace) + lw.tc_off : nullptr;
    tcb = lw.tc_bytes;
  } else {
    SB_TRY(tc_scratch_of(md, st, tcs, tcb));
  }
  TcPlan tp;
  const bool tc = tcs && tc_plan_for(md->lm_head, T, tp);
  if (T > kFusedNormMaxRows && !tc) {
    SB_TRY(run_norm(md, st, st->hidden, false, md->final_norm, s));
    p.pro = PRO_NONE;
    p.x = st->xnorm;
  }
  p.epi = EPI_ARGMAX;
  p.logits = st->logits;
  p.logits_mult = md->logits_mult;
  p.part_val = w.val;
  p.part_idx = w.idx;
  p.counter = w.counter;
  p.n_ctas = w.n_ctas;
  p.mode = st->mode;
  p.batch = st->batch;
  p.step = step;
  p.ids_io = st->ids;
  p.out_ids = st->out_ids;
  p.finished = st->finished;
  p.eos_id = st->eos_id;
  p.pad_id = st->pad_id;
  p.ctrl = st->ctrl;
  return run_linear(md->lm_head, p, tcs, tcb, st->use_pdl != 0, s);
}

// Whether the attention kernel writes the o-projection's tcgen05 operand
// itself (so the o GEMM runs without a preparation launch): the o projection
// takes the tensor-core GEMM with one token tile, and for fp8 its K split has
// one rank per KV head (each rank's 512 columns are one attention CTA's
// output, scaled by that CTA's own power of two); bf16 operands need no scale.
static bool o_operand_from_attn(const SbModel* md, const SbState* st, const SbLayer& L, void* tcs, TcPlan& tp) {
  const int T = st->batch * st->m;
  if (!tcs || !lin_ok(L.o) || !tc_plan_for(L.o, T, tp) || tp.mtiles != 1) return false;
  if (L.o.fmt != SB_FMT_FP8) return true;
  const int G = md->n_q / md->n_kv;
  return tp.split == md->n_kv && tp.kb % tp.split == 0 && tp.kb / tp.split == G;
}

static int launch_attention(const SbModel* md, const SbState* st, int l, cudaStream_t s) {
  const SbLayer& L = md->layers[l];
  AttnParams a;
  memset(&a, 0, sizeof(a));
  {
    size_t tcb = 0;
    void* tcs = nullptr;
    TcPlan tp;
    SB_TRY(tc_scratch_of(md, st, tcs, tcb));
    if (o_operand_from_attn(md, st, L, tcs, tp)) {
      const int T = st->batch * st->m;
      a.opnd = static_cast<uint8_t*>(tcs);
      a.opnd_shift = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(tcs) + tc_shift_offset(L.o.fmt, L.o.k, T));
      a.opnd_mp = tp.mp;
      a.opnd_np = tp.np;
      a.opnd_fp8 = L.o.fmt == SB_FMT_FP8 ? 1 : 0;
    }
  }
  a.q = st->q;
  a.k_cache = L.k_cache;
  a.v_cache = L.v_cache;
  a.out = st->attn;
  a.n_q = md->n_q;
  a.n_kv = md->n_kv;
  a.max_len = md->max_len;
  a.m_per = st->m;
  a.attn_mult = md->attn_mult;
  a.ctrl = st->ctrl;
  a.prompt_len = st->prompt_len;
  a.split = attn_split(st->batch * md->n_kv, md->max_len);
  a.chunk_cap = attn_key_capacity(md->max_len, a.split);
  const int tiles = a.chunk_cap / attn_tile_keys(a.split);  // K tiles per CTA at most (as many V tiles)
  a.slots = 2 * tiles < 3 ? 2 * tiles : 3;
  if (a.slots < 2) a.slots = 2;
  a.cache_rows = static_cast<long long>(md->max_batch) * md->n_kv * md->max_len;
  a.qblocks = 1;
  const int rc = attn_launch(a, st->batch, st->use_pdl != 0, s);
  if (rc == SB_ERR_CONFIG) return fail(rc, "no attention configuration (rows=%d)", (md->n_q / md->n_kv) * st->m);
  if (rc != 0) return fail(rc, "attention launch: %s", cudaGetErrorString((cudaError_t)rc));
  return 0;
}

// One kernel of the step: op = SB_OP_* for layer l.
static int launch_op(const SbModel* md, const SbState* st, int l, int op, int step, cudaStream_t s) {
  const int T = st->batch * st->m;
  const bool pdl = st->use_pdl != 0;
  if (op == SB_OP_LM_HEAD) {
    if (!lin_ok(md->lm_head)) return fail(SB_ERR_ARG, "bad lm_head");
    return launch_lm_head(md, st, step, s);
  }
  if (op == SB_OP_ATTN) return launch_attention(md, st, l, s);
  const SbLayer& L = md->layers[l];
  if (!lin_ok(L.qkv) || !lin_ok(L.o) || !lin_ok(L.gate_up) || !lin_ok(L.down))
    return fail(SB_ERR_ARG, "layer %d: bad packed linear", l);
  size_t tcb = 0;
  void* tcs = nullptr;
  WsLayout ws;
  SB_TRY(tc_scratch_of(md, st, tcs, tcb, &ws));
  const bool chain = ws.chain_off != 0;
  const ChainPlan& cp = ws.chain;
  ChainBufs cb;
  if (chain) chain_bufs(st, ws, cb);
  auto launch_bs = [&](const char* what, const GemvParams& p, const SbLinear& lin, const void* operand,
                       const TcPlan& pl) {
    const int rc = tc_launch_bs(p, lin.w_tc, operand, pl, pdl, s);
    if (rc != 0) return fail(rc, "tensor-core gemm launch (%s, block-scaled operand, n=%d k=%d m=%d): %s", what, p.n,
                             p.k, p.m, rc < 1000 ? cudaGetErrorString((cudaError_t)rc) : "config");
    return 0;
  };
  // the tensor-core path computes the RMSNorm prologue in its operand preparation
  auto sep_norm_for = [&](const SbLinear& lin) {
    TcPlan tp;
    return T > kFusedNormMaxRows && !(tcs && tc_plan_for(lin, T, tp));
  };
  if (op == SB_OP_QKV) {  // RMSNorm (layer 0: embedding x12) -> q/k/v -> RoPE + cache write
    GemvParams p = base_params(L.qkv, T);
    p.pro = l == 0 ? PRO_EMBED : PRO_RMSNORM;
    p.x = st->hidden;
    if (sep_norm_for(L.qkv)) {
      SB_TRY(run_norm(md, st, st->hidden, l == 0, L.in_norm, s));
      p.pro = PRO_NONE;
      p.x = st->xnorm;
    }
    p.norm_w = L.in_norm;
    p.eps = md->eps;
    p.ids = st->ids;
    p.embed = md->embed;
    p.embed_rows = md->vocab;
    p.emb_mult = md->emb_mult;
    p.hidden_out = st->hidden;
    p.epi = EPI_QKV;
    p.q_out = st->q;
    p.k_cache = L.k_cache;
    p.v_cache = L.v_cache;
    p.n_q = md->n_q;
    p.n_kv = md->n_kv;
    p.max_len = md->max_len;
    p.m_per = st->m;
    p.cos_tab = md->rope_cos;
    p.sin_tab = md->rope_sin;
    p.rope_max = md->rope_max_pos;
    p.rope_off = st->rope_off;
    p.ctrl = st->ctrl;
    if (chain && l > 0) {  // the previous layer's down GEMM wrote the operand and the norm statistics
      p.pro = PRO_NONE;
      p.x = nullptr;
      p.ssq_in = cb.ssq;
      return launch_bs("q/k/v", p, L.qkv, cb.op1, cp.qkv);
    }
    return run_linear(L.qkv, p, tcs, tcb, pdl, s);
  }
  if (op == SB_OP_O || op == SB_OP_DOWN) {  // o / down -> residual scale-add into hidden
    const SbLinear& lin = op == SB_OP_O ? L.o : L.down;
    GemvParams p = base_params(lin, T);
    p.pro = PRO_NONE;
    p.x = op == SB_OP_O ? st->attn : st->act;
    p.epi = EPI_RESID;
    p.y = st->hidden;
    p.res_mult = md->res_mult;
    if (chain) {
      if (op == SB_OP_O || l + 1 < md->n_layers) {  // write gate/up's operand, or the next layer's q/k/v's
        const TcPlan& nx = op == SB_OP_O ? cp.gu : cp.qkv;
        p.nx_op = cb.op1;
        p.nx_g = op == SB_OP_O ? L.post_norm : md->layers[l + 1].in_norm;
        p.nx_ssq = cb.ssq;
        p.nx_np = nx.np;
        p.nx_mp = nx.mp;
      }
      if (op == SB_OP_DOWN) return launch_bs("down", p, L.down, cb.op2, cp.down);  // gate/up wrote the operand
    }
    TcPlan tp;
    if (op == SB_OP_O && o_operand_from_attn(md, st, L, tcs, tp)) {  // the attention wrote the operand
      const size_t need = tc_operand_bytes(lin.fmt, lin.k, T);
      if (need > tcb) return fail(SB_ERR_ARG, "tensor-core operand scratch too small (%zu < %zu)", tcb, need);
      const int rc = tc_launch(p, lin.w_tc, tcs, tp, lin.fmt, pdl, s, true);
      if (rc != 0) return fail(rc, "tensor-core gemm launch (o, n=%d k=%d m=%d): %s", p.n, p.k, p.m,
                               rc < 1000 ? cudaGetErrorString((cudaError_t)rc) : "config");
      return 0;
    }
    return run_linear(lin, p, tcs, tcb, pdl, s);
  }
  // gate/up: RMSNorm -> interleaved gate|up -> SiLU(gate)*up
  if (chain) {  // o wrote the operand and the norm statistics; write down's operand
    GemvParams p = base_params(L.gate_up, T);
    p.eps = md->eps;
    p.ssq_in = cb.ssq;
    p.epi = EPI_SWIGLU;
    p.y = st->act;
    p.nx_op = cb.op2;
    p.nx_np = cp.down.np;
    p.nx_mp = cp.down.mp;
    return launch_bs("gate/up", p, L.gate_up, cb.op1, cp.gu);
  }
  GemvParams p = base_params(L.gate_up, T);
  p.pro = PRO_RMSNORM;
  p.x = st->hidden;
  p.norm_w = L.post_norm;
  p.eps = md->eps;
  if (sep_norm_for(L.gate_up)) {
    SB_TRY(run_norm(md, st, st->hidden, false, L.post_norm, s));
    p.pro = PRO_NONE;
    p.x = st->xnorm;
  }
  p.epi = EPI_SWIGLU;
  p.y = st->act;
  return run_linear(L.gate_up, p, tcs, tcb, pdl, s);
}

extern "C" {

const char* sb_last_error(void) { return g_err; }
uint64_t sb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }
int sb_version(void) { return 1; }

size_t sb_workspace_bytes(const SbModel* md, int32_t tokens) {
  if (!md || tokens < 1) return 0;
  return ws_layout(md, tokens).total;
}

size_t sb_decode_step_scratch_offset(const SbModel* md, int32_t tokens) {
  if (!md || tokens < 1) return static_cast<size_t>(-1);
  const WsLayout w = ws_layout(md, tokens);
  return w.step_bytes ? w.step_off : static_cast<size_t>(-1);
}

int32_t sb_decode_step_fused_ok(const SbModel* md, const SbState* st) {
  if (!md || !st || check_state(md, st) != 0) return 0;
  StepPlan pl;
  return step_plan(md, st, pl, nullptr) ? 1 : 0;
}

int sb_decode_step(const SbModel* md, const SbState* st, int32_t step, sb_stream_t stream) {
  return sb_decode_step_ex(md, st, step, 0, stream);
}

int sb_decode_step_ex(const SbModel* md, const SbState* st, int32_t step, int32_t flags, sb_stream_t stream) {
  SB_TRY(check_state(md, st));
  if (!md->layers || md->n_layers < 1) return fail(SB_ERR_ARG, "no layers");
  if ((flags & SB_STEP_PER_OP) && (flags & SB_STEP_FUSED)) return fail(SB_ERR_ARG, "conflicting step flags");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // flags 0: forwards of one stream (B = 1 decode, verify of <= 8 tokens) as
  // the fused step where it serves them (measured faster there on B200, 40
  // NVFP4 layers: 1.46 vs 1.49-1.53 ms per decode step, 4.04 vs 4.20 ms per
  // 8-token verify), everything else on the per-op kernels
  const bool fused_default = flags == 0 && st->batch == 1;
  if ((flags & SB_STEP_FUSED) || fused_default) {
    StepPlan pl;
    const char* why = "";
    if (step_plan(md, st, pl, &why)) {
      const WsLayout w = ws_layout(md, st->batch * st->m);
      if (st->workspace_bytes < w.total)
        return fail(SB_ERR_ARG, "workspace too small (%zu < %zu)", st->workspace_bytes, w.total);
      const int rc = step_launch(md, st, step, static_cast<char*>(st->workspace) + w.step_off, pl, s);
      if (rc != 0) return fail(rc, "fused step launch: %s", rc < 1000 ? cudaGetErrorString((cudaError_t)rc) : "config");
      return 0;
    }
    if (flags & SB_STEP_FUSED) return fail(SB_ERR_CONFIG, "the fused step does not serve this forward: %s", why);
  }
  for (int l = 0; l < md->n_layers; ++l)
    for (int op = SB_OP_QKV; op <= SB_OP_DOWN; ++op) SB_TRY(launch_op(md, st, l, op, step, s));
  return launch_op(md, st, 0, SB_OP_LM_HEAD, step, s);
}

int sb_decode_op(const SbModel* md, const SbState* st, int32_t layer, int32_t op, int32_t step, sb_stream_t stream) {
  SB_TRY(check_state(md, st));
  if (!md->layers || layer < 0 || layer >= md->n_layers) return fail(SB_ERR_ARG, "bad layer %d", layer);
  if (op < SB_OP_QKV || op > SB_OP_LM_HEAD) return fail(SB_ERR_ARG, "bad op %d", op);
  return launch_op(md, st, layer, op, step, static_cast<cudaStream_t>(stream));
}

int sb_lm_head_argmax(const SbModel* md, const SbState* st, int32_t step, sb_stream_t stream) {
  SB_TRY(check_state(md, st));
  return launch_op(md, st, 0, SB_OP_LM_HEAD, step, static_cast<cudaStream_t>(stream));
}

int sb_linear(const SbLinear* lin, const uint16_t* x, uint16_t* y, int32_t m, int32_t use_pdl, sb_stream_t stream) {
  return sb_linear_ex(lin, x, y, m, nullptr, 0, use_pdl, stream);
}

// sb_linear_ex runs the tensor-core GEMM on blocks of at most this many rows
// (one activation preparation + one launch each; weights re-streamed per block)
static const int kLinearBlockRows = 8192;

size_t sb_linear_workspace_bytes(const SbLinear* lin, int32_t m) {
  if (!lin || m < 1) return 0;
  return tc_scratch_need(*lin, m > kLinearBlockRows ? kLinearBlockRows : m);
}

int sb_linear_ex(const SbLinear* lin, const uint16_t* x, uint16_t* y, int32_t m, void* workspace,
                 size_t workspace_bytes, int32_t use_pdl, sb_stream_t stream) {
  if (!lin || !lin_ok(*lin) || !x || !y) return fail(SB_ERR_ARG, "sb_linear: bad arguments");
  if (m < 1) return fail(SB_ERR_ARG, "sb_linear: m must be >= 1");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TcPlan pl;
  if (workspace && tc_plan_for(*lin, m > kLinearBlockRows ? kLinearBlockRows : m, pl)) {
    // tensor-core path: token tiles of 128 inside one launch, blocks of kLinearBlockRows
    for (int r0 = 0; r0 < m; r0 += kLinearBlockRows) {
      const int mr = m - r0 < kLinearBlockRows ? m - r0 : kLinearBlockRows;
      GemvParams p = base_params(*lin, mr);
      p.pro = PRO_NONE;
      p.x = x + static_cast<size_t>(r0) * lin->k;
      p.epi = EPI_STORE;
      p.y = y + static_cast<size_t>(r0) * lin->n;
      SB_TRY(run_linear(*lin, p, mr > 8 ? workspace : nullptr, workspace_bytes, use_pdl != 0, s));
    }
    return 0;
  }
  GemvParams p = base_params(*lin, m);
  p.pro = PRO_NONE;
  p.x = x;
  p.epi = EPI_STORE;
  p.y = y;
  return run_small(*lin, p, use_pdl != 0, s);
}

// ---- native prefill -------------------------------------------------------------
// Query tokens per attention CTA (R = n_q / n_kv * 8 query rows <= 64) and the
// projection rows per launch (whole streams).
static const int kPrefillQBlock = 8;

// The prefill's attention runs on the two-pass prefill kernel
// (attention_pf.cu) where it serves the head grouping, else on the decode
// kernel with query blocks of kPrefillQBlock positions.
static const int kPrefillBlockRows = 8192;

static int prefill_streams_per_block(int B, int T) {
  int spb = kPrefillBlockRows / T;
  if (spb < 1) spb = 1;
  return spb < B ? spb : B;
}

struct PrefillWs {
  int32_t* ctrl;
  void* tc;
  size_t tc_bytes, total;
};
static PrefillWs prefill_ws(const SbModel* md, int B, int T, void* base) {
  PrefillWs w;
  const int rows = prefill_streams_per_block(B, T) * T;
  size_t need = 0;
  for (int l = 0; md->layers && l < md->n_layers; ++l) {
    const SbLayer& L = md->layers[l];
    const SbLinear* lins[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
    for (const SbLinear* x : lins) {
      const size_t b = tc_scratch_need(*x, rows);
      if (b > need) need = b;
    }
  }
  w.ctrl = static_cast<int32_t*>(base);
  w.tc = base ? static_cast<char*>(base) + 256 : nullptr;
  w.tc_bytes = need;
  w.total = 256 + need;
  return w;
}

// A prefill block of `rows` token rows runs each projection on the tcgen05
// GEMM (tile copy present and the shape served), else on the GEMV kernels,
// which compute every fused epilogue (RoPE + cache write, SwiGLU, residual)
// for up to 64 rows in one launch (one row chunk per CTA).
static const int kPrefillGemvMaxRows = 64;
static bool prefill_rows_served(const SbLinear& l, int rows) {
  TcPlan pl;
  return rows <= kPrefillGemvMaxRows || tc_plan_for(l, rows, pl);
}

static int check_prefill(const SbModel* md, int B, int T) {
  if (!md || !md->layers || md->n_layers < 1) return fail(SB_ERR_ARG, "sb_prefill: no model");
  if (B < 1 || B > md->max_batch) return fail(SB_ERR_ARG, "sb_prefill: batch %d outside [1, %d]", B, md->max_batch);
  if (T < kPrefillQBlock || T % kPrefillQBlock || T > md->max_len)
    return fail(SB_ERR_ARG, "sb_prefill: T=%d must be a multiple of %d and <= max_len %d", T, kPrefillQBlock,
                md->max_len);
  if (md->head_dim != 128 || md->n_q % md->n_kv || (md->n_q / md->n_kv) * kPrefillQBlock > 64)
    return fail(SB_ERR_CONFIG, "sb_prefill: needs head_dim 128 and n_q / n_kv <= 8");
  // the blocks are spb streams each, the last one batch % spb streams if not zero
  const int spb = prefill_streams_per_block(B, T);
  const int rows = spb * T, tail = (B % spb) * T;
  for (int l = 0; l < md->n_layers; ++l) {
    const SbLayer& L = md->layers[l];
    const SbLinear* lins[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
    for (const SbLinear* x : lins) {
      if (!lin_ok(*x)) return fail(SB_ERR_ARG, "sb_prefill: layer %d: bad packed linear", l);
      if (!prefill_rows_served(*x, rows) || (tail && !prefill_rows_served(*x, tail)))
        return fail(SB_ERR_CONFIG, "sb_prefill: layer %d: blocks of %d / %d rows need the tensor-core tile copy "
                    "of every projection (more than %d rows)", l, rows, tail, kPrefillGemvMaxRows);
    }
  }
  return 0;
}

extern "C" size_t sb_prefill_workspace_bytes(const SbModel* md, int32_t batch, int32_t T) {
  if (!md || batch < 1 || T < 1) return 0;
  return prefill_ws(md, batch, T, nullptr).total;
}

extern "C" int32_t sb_prefill_block_rows(const SbModel* md, int32_t batch, int32_t T) {
  if (!md || batch < 1 || T < 1) return 0;
  return prefill_streams_per_block(batch, T) * T;
}

extern "C" int sb_prefill(const SbModel* md, uint16_t* hidden, int32_t batch, int32_t T, const int32_t* prompt_len,
                          uint16_t* q, uint16_t* attn, uint16_t* act, void* workspace, size_t workspace_bytes,
                          sb_stream_t stream) {
  SB_TRY(check_prefill(md, batch, T));
  if (!hidden || !q || !attn || !act || !workspace) return fail(SB_ERR_ARG, "sb_prefill: buffer missing");
  const PrefillWs ws = prefill_ws(md, batch, T, workspace);
  if (workspace_bytes < ws.total)
    return fail(SB_ERR_ARG, "sb_prefill: workspace too small (%zu < %zu)", workspace_bytes, ws.total);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int H = md->hidden, NQ = md->n_q * 128, spb = prefill_streams_per_block(batch, T);
  const size_t head_rows = static_cast<size_t>(md->n_kv) * md->max_len * 128;  // cache elements per stream
  const size_t tcb = workspace_bytes - 256;
  SB_TRY(set_ctrl_launch(ws.ctrl, 0, T, s));
  for (int l = 0; l < md->n_layers; ++l) {
    const SbLayer& L = md->layers[l];
    // q/k/v: RMSNorm prologue, RoPE (positions 0..T-1) + K/V written to cache slots 0..T-1
    for (int b0 = 0; b0 < batch; b0 += spb) {
      const int nb = batch - b0 < spb ? batch - b0 : spb;
      const size_t r0 = static_cast<size_t>(b0) * T;
      GemvParams p = base_params(L.qkv, nb * T);
      p.pro = PRO_RMSNORM;
      p.x = hidden + r0 * H;
      p.norm_w = L.in_norm;
      p.eps = md->eps;
      p.epi = EPI_QKV;
      p.q_out = q + r0 * NQ;
      p.k_cache = L.k_cache + b0 * head_rows;
      p.v_cache = L.v_cache + b0 * head_rows;
      p.n_q = md->n_q;
      p.n_kv = md->n_kv;
      p.max_len = md->max_len;
      p.m_per = T;
      p.cos_tab = md->rope_cos;
      p.sin_tab = md->rope_sin;
      p.rope_max = md->rope_max_pos;
      p.ctrl = ws.ctrl;
      p.row_len = prompt_len;  // token tiles entirely in padding are skipped
      p.row_T = T;
      p.row_b0 = b0;
      SB_TRY(run_linear(L.qkv, p, ws.tc, tcb, false, s));
    }
    // causal attention over the right-padded prompts: query blocks of kPrefillQBlock tokens
    AttnParams a;
    memset(&a, 0, sizeof(a));
    a.q = q;
    a.k_cache = L.k_cache;
    a.v_cache = L.v_cache;
    a.out = attn;
    a.n_q = md->n_q;
    a.n_kv = md->n_kv;
    a.max_len = md->max_len;
    a.m_per = kPrefillQBlock;
    a.qblocks = T / kPrefillQBlock;
    a.attn_mult = md->attn_mult;
    a.ctrl = ws.ctrl;
    a.prompt_len = prompt_len;
    a.split = 1;
    a.chunk_cap = attn_key_capacity(T, 1);
    a.slots = 2;
    a.cache_rows = static_cast<long long>(md->max_batch) * md->n_kv * md->max_len;
    const int rc = attn_prefill_ok(md->n_q, md->n_kv) ? attn_prefill_launch(a, batch, T, s)
                                                                           : attn_launch(a, batch, false, s);
    if (rc == SB_ERR_CONFIG) return fail(rc, "sb_prefill: no attention configuration for T=%d", T);
    if (rc != 0) return fail(rc, "sb_prefill: attention launch: %s", cudaGetErrorString((cudaError_t)rc));
    // per block of streams: o (+ residual), gate/up (RMSNorm, SwiGLU), down (+ residual)
    for (int b0 = 0; b0 < batch; b0 += spb) {
      const int nb = batch - b0 < spb ? batch - b0 : spb;
      const size_t r0 = static_cast<size_t>(b0) * T;
      auto padding = [&](GemvParams& g) {
        g.row_len = prompt_len;
        g.row_T = T;
        g.row_b0 = b0;
      };
      GemvParams p = base_params(L.o, nb * T);
      p.pro = PRO_NONE;
      p.x = attn + r0 * NQ;
      p.epi = EPI_RESID;
      p.y = hidden + r0 * H;
      p.res_mult = md->res_mult;
      padding(p);
      SB_TRY(run_linear(L.o, p, ws.tc, tcb, false, s));
      p = base_params(L.gate_up, nb * T);
      p.pro = PRO_RMSNORM;
      p.x = hidden + r0 * H;
      p.norm_w = L.post_norm;
      p.eps = md->eps;
      p.epi = EPI_SWIGLU;
      p.y = act;
      padding(p);
      SB_TRY(run_linear(L.gate_up, p, ws.tc, tcb, false, s));
      p = base_params(L.down, nb * T);
      p.pro = PRO_NONE;
      p.x = act;
      p.epi = EPI_RESID;
      p.y = hidden + r0 * H;
      p.res_mult = md->res_mult;
      padding(p);
      SB_TRY(run_linear(L.down, p, ws.tc, tcb, false, s));
    }
  }
  return 0;
}

int sb_dequant_f32(const SbLinear* lin, float* out, sb_stream_t stream) {
  if (!lin || !lin_ok(*lin) || !out) return fail(SB_ERR_ARG, "sb_dequant_f32: bad arguments");
  SB_TRY(dequant_launch(*lin, out, true, static_cast<cudaStream_t>(stream)));
  return 0;
}

int sb_dequant_bf16(const SbLinear* lin, uint16_t* out, sb_stream_t stream) {
  if (!lin || !lin_ok(*lin) || !out) return fail(SB_ERR_ARG, "sb_dequant_bf16: bad arguments");
  SB_TRY(dequant_launch(*lin, out, false, static_cast<cudaStream_t>(stream)));
  return 0;
}

int sb_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int32_t rows, int32_t n, float eps, sb_stream_t s) {
  if (!x || !w || !y || rows < 1 || n < 1) return fail(SB_ERR_ARG, "sb_rmsnorm: bad arguments");
  SB_TRY(rmsnorm_launch(x, w, y, rows, n, eps, static_cast<cudaStream_t>(s)));
  return 0;
}

int sb_silu_mul(const uint16_t* g, const uint16_t* u, uint16_t* o, int64_t count, sb_stream_t s) {
  if (!g || !u || !o || count < 0) return fail(SB_ERR_ARG, "sb_silu_mul: bad arguments");
  if (count == 0) return 0;
  SB_TRY(silu_mul_launch(g, u, o, count, static_cast<cudaStream_t>(s)));
  return 0;
}

int sb_residual_scale(const uint16_t* x, const uint16_t* y, uint16_t* z, int64_t count, float alpha, sb_stream_t s) {
  if (!x || !y || !z || count < 0) return fail(SB_ERR_ARG, "sb_residual_scale: bad arguments");
  if (count == 0) return 0;
  SB_TRY(residual_launch(x, y, z, count, alpha, static_cast<cudaStream_t>(s)));
  return 0;
}

int sb_rope(uint16_t* x, int32_t rows, int32_t heads, const int32_t* pos, const uint16_t* cs, const uint16_t* sn,
            sb_stream_t s) {
  if (!x || !pos || !cs || !sn || rows < 1 || heads < 1) return fail(SB_ERR_ARG, "sb_rope: bad arguments");
  SB_TRY(rope_launch(x, rows, heads, pos, cs, sn, static_cast<cudaStream_t>(s)));
  return 0;
}

int sb_argmax_bf16(const uint16_t* x, int32_t rows, int32_t n, int64_t* out, sb_stream_t s) {
  if (!x || !out || rows < 1 || n < 1) return fail(SB_ERR_ARG, "sb_argmax_bf16: bad arguments");
  SB_TRY(argmax_launch(x, rows, n, out, static_cast<cudaStream_t>(s)));
  return 0;
}

int sb_attention(const SbModel* md, const SbState* st, int32_t layer, sb_stream_t stream) {
  SB_TRY(check_state(md, st));
  if (layer < 0 || layer >= md->n_layers) return fail(SB_ERR_ARG, "bad layer");
  return launch_attention(md, st, layer, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// lm_head + argmax without a caller-provided workspace.
//
// Some callers cannot allocate device memory: an embedding runtime that binds
// only this C ABI and owns no device allocator, or a latency-critical serving
// loop that forbids cudaMalloc because it synchronises the whole device and
// may fail once another framework has reserved the HBM pool.  This variant of
// sb_lm_head_argmax keeps the lm_head launch's scratch (argmax partials,
// completion counter and, on the tensor-core path, the lm_head's activation
// operand) in a fixed file-scope device array instead of state->workspace,
// which may be NULL.  The array is kStaticLmScratchBytes (256 KiB) and lives
// on every GPU that loads this library until the process exits.  Calls whose
// lm_head scratch would not fit are rejected.  All calls share the array, so
// two calls that overlap on the GPU (different streams, or two processes'
// kernels interleaved through one context) race: serialise them.
// ---------------------------------------------------------------------------
namespace {
constexpr size_t kStaticLmScratchBytes = 256 * 1024;
__device__ __align__(256) unsigned char g_lm_scratch[kStaticLmScratchBytes];
constexpr int kMaxDevices = 64;
// device address of g_lm_scratch per device, looked up once per device
std::atomic<void*> g_lm_scratch_addr[kMaxDevices] = {};
}  // namespace

extern "C" int sb_lm_head_argmax_static(const SbModel* md, const SbState* st, int32_t step, sb_stream_t stream) {
  SB_TRY(check_state(md, st, false));
  if (!lin_ok(md->lm_head)) return fail(SB_ERR_ARG, "bad lm_head");
  const int T = st->batch * st->m;
  const size_t need = lm_layout(md, T).total;
  if (need > kStaticLmScratchBytes)
    return fail(SB_ERR_CONFIG,
                "sb_lm_head_argmax_static: %d token rows need %zu lm_head scratch bytes, more than the fixed %zu; "
                "use sb_lm_head_argmax with a caller workspace",
                T, need, kStaticLmScratchBytes);
  int dev = 0;
  SB_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(SB_ERR_ARG, "device index %d out of range", dev);
  // one-time set-up per device (this device is current): host code must use
  // the symbol's device address, never &g_lm_scratch, which is a host stand-in.
  // Two threads racing here both store the same address.
  void* base = g_lm_scratch_addr[dev].load(std::memory_order_acquire);
  if (!base) {
    const cudaError_t e = cudaGetSymbolAddress(&base, g_lm_scratch);
    if (e != cudaSuccess) return fail(e, "cudaGetSymbolAddress(g_lm_scratch): %s", cudaGetErrorString(e));
    g_lm_scratch_addr[dev].store(base, std::memory_order_release);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the completion counter (first 256 bytes) must start at zero on every call
  SB_TRY(cudaMemsetAsync(base, 0, 256, s));
  SbState local = *st;
  local.workspace = base;
  local.workspace_bytes = kStaticLmScratchBytes;
  return launch_lm_head(md, &local, step, s, true);
}
