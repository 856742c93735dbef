// Fused decode step for up to 8 token rows: one cooperative launch per
// forward.  See step.cu for the kernel and the design notes.
#pragma once
#include "gemv.cuh"

namespace sb {

constexpr int kStepMaxLayers = 64;
constexpr int kStepKeys = 32;       // keys per attention split at most
constexpr int kStepMaxSplit = 32;   // attention splits per (stream, KV head) at most
constexpr int kStepMaxRows = 32;    // query rows per KV head (query heads per KV head x tokens)

// Per-layer pointers (mat: 0 = qkv, 1 = o, 2 = gate_up, 3 = down).
struct StepLayer {
  const uint16_t* in_norm;
  const uint16_t* post_norm;
  const uint8_t* w[4];
  const uint8_t* s[4];
  float g[4];
  uint16_t* k_cache;
  uint16_t* v_cache;
};

struct StepParams {
  // model
  int n_layers, hidden, inter, n_q, n_kv, vocab, max_len, rope_max;
  int n_tiles[5];  // 16-row tiles of qkv, o, gate_up, down, lm_head
  int n_rows[5];   // logical rows of the same
  float eps, attn_mult, emb_mult, res_mult, logits_mult;
  const uint16_t* embed;
  const uint16_t* final_norm;
  const uint16_t* cos_tab;
  const uint16_t* sin_tab;
  const uint8_t* lm_w;
  const uint8_t* lm_s;
  float lm_g;
  // forward state
  int batch, m_per, M, mode, step;
  int64_t* ids;
  int32_t* ctrl;
  const int32_t* prompt_len;
  const int32_t* rope_off;
  int32_t* finished;
  int64_t* out_ids;
  uint16_t* resid;  // [M][hidden] residual stream
  uint16_t* q;
  uint16_t* attn;
  uint16_t* act;
  uint16_t* logits;
  int64_t eos_id, pad_id;
  // scratch (state workspace): counters, attention statistics and partial
  // outputs, argmax partials
  unsigned* sync;
  // activations handed between CTAs as 8-byte words {2 bf16, epoch}: a
  // reader polls the words themselves (no barrier between the phases)
  unsigned long long* ll_h;     // residual stream [M][hidden/2]
  unsigned long long* ll_q;     // q rows [M][n_q*64]
  unsigned long long* ll_kv;    // this forward's k and v rows [M][n_kv][2][64]
  unsigned long long* ll_attn;  // attention output [M][n_q*64]
  unsigned long long* ll_act;   // SwiGLU output [M][inter/2]
  float2* attn_stats;  // [B*n_kv][n_split][R]
  float* attn_part;    // [B*n_kv][n_split][R][128]
  float* am_val;       // [grid][M]
  int* am_idx;
  int n_split;
  int ring_bytes;
  int rounds_per_batch;
  int act_bytes;
  int rc_rows;  // residual rows cached per CTA (ceil(hidden tiles / grid) * 16)
  int inflight_cap;  // weight bytes in flight per CTA at most
  StepLayer layers[kStepMaxLayers];
};

// sync[] words: grid barrier count, argmax arrivals, the launch sequence
// number (epochs of the handed-over words), then per (stream, KV head) the
// statistics counter and the combine counter.
constexpr int kSyncGrid = 0;
constexpr int kSyncArgmax = 1;
constexpr int kSyncSeq = 2;
constexpr int kSyncStats = 64;
constexpr int kSyncCombine = 64 + 1024;
constexpr int kSyncWords = 64 + 2048;

// Warp slices of a projection with K inputs: wt warps per 16-row tile, kw K
// elements per warp (a whole number of kgroups; two tiles per round of 16
// warps when K has fewer than 16 kgroups).
__host__ __device__ constexpr int step_kgroup_elems(int fmt) {
  return fmt == SB_FMT_NVFP4 ? 64 : (fmt == SB_FMT_BF16 ? 16 : 32);
}
__host__ __device__ constexpr int step_wt(int fmt, int K) {
  return K / step_kgroup_elems(fmt) >= 16 ? 16 : K / step_kgroup_elems(fmt);
}
// f16 activation slices of one projection: [wt][M][kw + 8]
__host__ __device__ constexpr size_t step_act_bytes(int fmt, int K, int M) {
  return static_cast<size_t>(step_wt(fmt, K)) * M * (K / step_wt(fmt, K) + 8) * 2;
}

// Shared-memory layout, computed identically on the host and in the kernel.
// The projection buffers (activation slices, partials) and the attention
// buffers are never live at once and share one region.
struct StepLayout {
  size_t bars, endv, ss, shift, best, bval, flag, sp, rope, rc, un;
  size_t xs, red, tot;  // projections
  size_t aq, asc;       // attention
  size_t total;
};
__host__ __device__ inline StepLayout step_layout(size_t ring_bytes, int M, int R, int rounds_per_batch,
                                                  size_t act_bytes, int rc_rows) {
  auto up16 = [](size_t x) { return (x + 15) & ~size_t(15); };
  StepLayout L;
  L.bars = ring_bytes;                     // full[32], empty[32] mbarriers
  L.endv = L.bars + 64 * 8;                // producer: ring end and bytes of each entry in flight
  L.ss = up16(L.endv + 64 * 4);            // [16 warps][8 tokens]
  L.shift = up16(L.ss + 16 * 8 * 4);
  L.best = up16(L.shift + 16 * 8 * 4);
  L.bval = up16(L.best + 8 * 4);
  L.flag = up16(L.bval + 8 * 4);
  L.sp = up16(L.flag + 16);
  L.rope = up16(L.sp + sizeof(GemvParams));                  // [M][cos 64 | sin 64]
  L.rc = up16(L.rope + static_cast<size_t>(M) * 256);        // [M][rc_rows] residual rows of this CTA
  L.un = up16(L.rc + static_cast<size_t>(M) * rc_rows * 2);
  L.xs = L.un;
  L.red = up16(L.xs + act_bytes);          // [rounds][16 warps][16 rows][M]
  L.tot = up16(L.red + static_cast<size_t>(rounds_per_batch) * 16 * 16 * M * 4);
  const size_t proj_end = up16(L.tot + static_cast<size_t>(rounds_per_batch) * 2 * 16 * M * 4);
  L.aq = L.un;                                                // q rows [R][128] bf16
  L.asc = up16(L.aq + static_cast<size_t>(R) * 256);          // scores / p [R][32]
  const size_t attn_end = up16(L.asc + static_cast<size_t>(R) * kStepKeys * 4);
  L.total = proj_end > attn_end ? proj_end : attn_end;
  return L;
}

struct StepPlan {
  int fmt, n_split, rows, rounds_per_batch, ring_bytes, grid;
  size_t act_bytes, smem;
  int rc_rows;
};
// Whether the fused step serves (model, state); why = reason when not.
bool step_plan(const SbModel* md, const SbState* st, StepPlan& pl, const char** why);
size_t step_ws_bytes(const SbModel* md, int tokens);
int step_launch(const SbModel* md, const SbState* st, int step, void* ws, const StepPlan& pl, cudaStream_t stream);

}  // namespace sb
