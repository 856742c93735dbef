/*
 * starling_b200 -- C ABI of the B200 (sm_100a) Granite greedy-decode library.
 *
 * The reference (sims1253/starling) is pure Python: its decode step is a
 * Python loop over HF Granite modules, cuBLAS GEMMs (nn.Linear) and four
 * Triton glue kernels, captured into CUDA graphs.  Each entry point below
 * replaces one of those call sites; the reference location is cited beside
 * it.  Conventions:
 *
 *   - every pointer is a device pointer unless its comment says "host";
 *   - bf16 tensors are passed as uint16_t*; token ids are int64 like the
 *     reference's static_input_ids (llm_mega.py:123);
 *   - every call is asynchronous on `stream`, allocates nothing, never
 *     synchronises and never reads host memory after it returns, so it can be
 *     captured into a CUDA graph;
 *   - every call returns 0 on success, else an SB_ERR_* code or a
 *     cudaError_t value; sb_last_error() gives the message.
 */
#ifndef STARLING_B200_H
#define STARLING_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* sb_stream_t; /* a cudaStream_t */

/* error codes (cudaError_t values pass through unchanged; ours start at 1000) */
#define SB_OK 0
#define SB_ERR_ARG 1001     /* bad shape / pointer / format */
#define SB_ERR_CONFIG 1002  /* shape not supported by any kernel configuration */

/* weight formats (weight-only; activations stay bf16) */
#define SB_FMT_BF16 0  /* bf16 weights, as nn.Linear holds them */
#define SB_FMT_FP8 1   /* e4m3 + fp32 per-output-row scale */
#define SB_FMT_INT8 2  /* symmetric int8 + fp32 per-output-row scale */
#define SB_FMT_NVFP4 3 /* e2m1 + e4m3 scale per 16 K-elements + fp32 tensor scale */

/*
 * One packed linear layer y = x W^T (W logical [n, k]).  Packed layout
 * (written by starling_b200/pack.py): rows padded to n_pad = ceil(n/16)*16;
 * w = [n_pad/16 row tiles][k / kg kgroups][32 lanes][16 bytes], where a
 * kgroup is 64 (nvfp4), 32 (fp8/int8) or 16 (bf16) K elements and each lane's
 * 16 bytes are its mma.m16n8k16 A-fragments for those K elements.
 * scale: fp8/int8 -> float[n_pad]; nvfp4 -> e4m3 bytes
 * [n_pad/16][k/64][8 row pairs][8] ; bf16 -> NULL.
 *
 * w_tc (optional, fp8 and bf16): a second copy of the same rows (same packed
 * row order, same scale) for the tcgen05 GEMM that serves 9..128 token rows:
 * [ceil(n/128) tiles][k*eb/128 K blocks][16 row groups][8 K chunks][8 rows]
 * [16 bytes] (eb = bytes per element), i.e. every 128-row x 128-byte block is
 * contiguous in the no-swizzle K-major canonical layout of tcgen05.mma;
 * rows >= n are zero.  NULL: those token counts use the mma.sync GEMV.
 *
 * w_bs (optional, nvfp4 only): the block-scaled tensor-core copy used for 1..8
 * token rows (tcgen05.mma kind::mxf4nvf4): per (128-row tile, 256-element K
 * block) 18432 bytes = 16384 bytes of e2m1 codes (two per byte, lower K index
 * in the low nibble) laid out like w_tc (byte (row, kbyte) at rg*1024 +
 * kc*128 + r*16 + b), then the block scales as four 512-byte chunks, chunk j
 * covering K elements 64j..64j+63 of the block, byte (r % 32)*16 + (r / 32)*4
 * + i for tile row r and 16-element block i of the chunk.  Same packed row
 * order and tensor scale as w; rows >= n are zero.  K must be a multiple of
 * 256.  NULL: 1..8 rows use the mma.sync GEMV.
 */
typedef struct SbLinear {
  int32_t fmt;
  int32_t n;
  int32_t k;
  int32_t n_pad;
  const void* w;
  const void* scale;
  float global_scale; /* nvfp4 per-tensor scale, else 1 */
  int32_t _pad;
  const void* w_tc;
  const void* w_bs;
} SbLinear;

/* One decoder layer.  qkv rows are [q heads | k heads | v heads] with the
 * two RoPE halves of every q/k head interleaved (packed row 2j = dim j,
 * 2j+1 = dim j+64); gate_up rows interleave gate row i (2i) and up row i
 * (2i+1).  Caches are [max_batch, n_kv, max_len, 128] bf16, the StaticLayer
 * layout (transformers cache_utils.py:286-295). */
typedef struct SbLayer {
  const uint16_t* in_norm;
  const uint16_t* post_norm;
  SbLinear qkv;
  SbLinear o;
  SbLinear gate_up;
  SbLinear down;
  uint16_t* k_cache;
  uint16_t* v_cache;
} SbLayer;

typedef struct SbModel {
  int32_t hidden, n_q, n_kv, head_dim, inter, vocab, n_layers;
  int32_t max_len;    /* static cache length (max_cache_len) */
  int32_t max_batch;  /* cache batch dimension */
  int32_t rope_max_pos;
  float eps, attn_mult, emb_mult, res_mult, logits_mult; /* logits_mult = 1/logits_scaling */
  const uint16_t* embed;      /* bf16 [vocab, hidden] (tied with lm_head) */
  const uint16_t* final_norm; /* bf16 [hidden] */
  const uint16_t* rope_cos;   /* bf16 [rope_max_pos, 64]: cos(pos * inv_freq[j]) */
  const uint16_t* rope_sin;
  SbLinear lm_head;
  const SbLayer* layers; /* HOST array of n_layers */
} SbModel;

/* Per-forward state.  All dynamic values live in device memory so one
 * captured graph serves every replay. */
#define SB_CTRL_SLOT 0    /* cache slot of token 0 of the next forward */
#define SB_CTRL_PADLEN 1  /* padded prompt length T (right-padded batches) */
#define SB_CTRL_ACCEPT 2  /* verify: accepted prefix length (output) */
#define SB_CTRL_ERR 3     /* set non-zero by a kernel whose bounded wait expired (results invalid):
                             1 = decode GEMV, 2 = tensor-core GEMM, 3 = attention, 4 = fused step */
#define SB_CTRL_WORDS 8

#define SB_MODE_DECODE 0  /* argmax -> out_ids[step], feed back to ids, slot += M */
#define SB_MODE_VERIFY 1  /* argmax per token -> out_ids[0..M), accept length vs ids[1..M) */
#define SB_MODE_FIRST 2   /* as DECODE without advancing the slot (prefill's first token) */

typedef struct SbState {
  int32_t batch;    /* B streams */
  int32_t m;        /* tokens per stream in this forward (1 = decode, L = verify) */
  int32_t mode;     /* SB_MODE_* */
  int32_t use_pdl;  /* launch with programmatic dependent launch */
  int64_t eos_id;
  int64_t pad_id;
  int64_t* ids;             /* [B*m] input token ids */
  int32_t* ctrl;            /* [SB_CTRL_WORDS] */
  const int32_t* prompt_len; /* [B] real prompt lengths, or NULL (no padding) */
  const int32_t* rope_off;   /* [B] RoPE position offset (T - T_b), or NULL */
  int32_t* finished;         /* [B] EOS flags (batched decode), or NULL */
  int64_t* out_ids;          /* DECODE: [steps][B]; VERIFY: [m] */
  uint16_t* hidden;  /* [B*m, hidden] residual stream */
  uint16_t* q;       /* [B*m, n_q*128] */
  uint16_t* attn;    /* [B*m, n_q*128] */
  uint16_t* act;     /* [B*m, inter] */
  uint16_t* xnorm;   /* [B*m, hidden] normalised rows (used when B*m > 8) */
  uint16_t* logits;  /* [B*m, vocab] or NULL */
  void* workspace;   /* scratch, >= sb_workspace_bytes() bytes, zeroed once */
  size_t workspace_bytes;
} SbState;

/* ---- library ------------------------------------------------------------ */
const char* sb_last_error(void);
int sb_version(void);
/* kernels this library has launched so far in this process (host counter; a
 * launch recorded into a CUDA graph counts once, at capture) */
uint64_t sb_launch_count(void);
/* scratch bytes an SbState needs for (model, batch*m tokens) */
size_t sb_workspace_bytes(const SbModel* model, int32_t tokens);

/* Which kernel serves NVFP4 linears of 1..8 token rows whose SbLinear has a
 * w_bs copy (process-wide; no counterpart in the reference, whose NVFP4 path
 * is eager torch).  SB_NVFP4_AUTO (default): the block-scaled tcgen05 kernel where it measured faster on B200 -- matrices of
 * >= 256 row tiles (lm_head) at any row count and every 8-row forward -- else
 * the mma.sync GEMV; SB_NVFP4_BLOCK_SCALED: the block-scaled
 * kernel for every shape it serves; SB_NVFP4_MMA_SYNC: always the GEMV.
 * Decided when a launch is issued (a captured graph keeps the kernels it
 * recorded); workspaces from sb_workspace_bytes fit every choice.  Returns the
 * previous mode, or SB_ERR_ARG. */
#define SB_NVFP4_AUTO 0
#define SB_NVFP4_BLOCK_SCALED 1
#define SB_NVFP4_MMA_SYNC 2
int32_t sb_set_nvfp4_path(int32_t mode);

/* ---- fused decode step ---------------------------------------------------
 * One full forward of state->m new tokens per stream through every layer,
 * lm_head and argmax, i.e. FusedLLMMega._decode_step_eager
 * (src/starling/granite/llm_mega.py:493-589) plus the in-graph argmax /
 * feedback / position advance of MultiStepLLMMega._captured_step
 * (src/starling/granite/multistep.py:157-188); with m > 1 it is the verify
 * forward SpeculativeDecoder._verify_step_fused (speculative.py:598-680) with
 * the acceptance compare of speculative.py:430-459 fused on device.
 * `step` indexes out_ids in DECODE mode.  Forwards of one stream (batch 1:
 * B = 1 decode, verify of up to 8 tokens) run as the one-launch fused step
 * where it serves them (see sb_decode_step_ex), every other forward as about
 * 5 launches per layer. */
int sb_decode_step(const SbModel* model, const SbState* state, int32_t step, sb_stream_t stream);

/* sb_decode_step with the kernel path chosen by the caller:
 * flags = 0: as sb_decode_step; SB_STEP_PER_OP: the per-op kernels;
 * SB_STEP_FUSED: forwards of up to 8 token rows (batch * m) as ONE
 * cooperative launch (weights streamed through shared memory across layers,
 * activations handed between CTAs through flagged words; needs one weight
 * format for every projection, hidden / inter 2048 / 8192 or 512 / 1024,
 * max_len <= 1024 and batch * n_kv * ceil(max_len / 32) <= SMs), or
 * SB_ERR_CONFIG where it does not serve the forward.  No reference counterpart (choice between the two paths). */
#define SB_STEP_PER_OP 1
#define SB_STEP_FUSED 2
int sb_decode_step_ex(const SbModel* model, const SbState* state, int32_t step, int32_t flags, sb_stream_t stream);
/* 1 when the fused step serves (model, state), else 0 */
int32_t sb_decode_step_fused_ok(const SbModel* model, const SbState* state);
/* byte offset inside an SbState workspace of the fused step's scratch (32-bit
 * words: [0..63] step counters, [64..1087] per (stream, KV head) attention
 * counters; all zero between forwards except word 2, a sequence number), or
 * SIZE_MAX when (model, tokens) has none */
size_t sb_decode_step_scratch_offset(const SbModel* model, int32_t tokens);

/* Launch ONE kernel of the decode step on its own (profiling / live timing
 * of a single kernel with the step's exact configuration): op = SB_OP_*,
 * layer ignored for SB_OP_LM_HEAD.  Where the o projection runs on the
 * tensor-core GEMM (9..128 token rows) the attention launch writes its
 * activation operand, so SB_OP_O computes from what the last SB_OP_ATTN of
 * the same state and token count wrote.  With fp8 weights at 9..64 token
 * rows the o, gate/up and down launches likewise write the next
 * projection's operand (and, after a residual, the next RMSNorm's
 * statistics): SB_OP_GATE_UP computes from what the last SB_OP_O wrote,
 * SB_OP_DOWN from the last SB_OP_GATE_UP, SB_OP_QKV of layers > 0 from the
 * last SB_OP_DOWN.  No reference counterpart (the reference step has no
 * separable kernels of this kind). */
#define SB_OP_QKV 0
#define SB_OP_ATTN 1
#define SB_OP_O 2
#define SB_OP_GATE_UP 3
#define SB_OP_DOWN 4
#define SB_OP_LM_HEAD 5
int sb_decode_op(const SbModel* model, const SbState* state, int32_t layer, int32_t op, int32_t step,
                 sb_stream_t stream);

/* final RMSNorm + lm_head + argmax over state->hidden (B rows, before the
 * final norm): the prefill tail `lm_head(norm(hidden))/logits_scaling` +
 * `.argmax(-1)` (llm_mega.py:200-202, batched.py:275-276). */
int sb_lm_head_argmax(const SbModel* model, const SbState* state, int32_t step, sb_stream_t stream);

/* sb_lm_head_argmax for callers that cannot allocate device memory (no
 * device allocator of their own, or cudaMalloc forbidden because it
 * synchronises the device).  No counterpart in the reference.  Same inputs
 * and outputs as sb_lm_head_argmax; state->workspace is ignored and may be
 * NULL: the scratch is a fixed 256 KiB device array inside the library (held
 * on every GPU that loads it until exit).  Only the lm_head launch's own
 * scratch must fit (its argmax partials, plus its activation operand when the
 * lm_head runs on the tensor-core GEMM); calls where it would not return
 * SB_ERR_CONFIG.  The first call on a device looks up the array's device
 * address; make that first call before any stream capture.  Calls share the
 * array: calls that overlap on the GPU race. */
int sb_lm_head_argmax_static(const SbModel* model, const SbState* state, int32_t step, sb_stream_t stream);

/* ---- speculative decoding loop on the device -------------------------------
 * The verify / accept loop of SpeculativeDecoder.generate
 * (src/starling/granite/speculative.py:400-539) as ONE CUDA graph: a setup
 * kernel, then WHILE (continue) { SWITCH (k - 1) { the verify forward of
 * [last emitted token, draft[draft_pos : draft_pos + k]] (sb_decode_step on
 * verify[k - 1]) } ; control kernel }.  The control kernel applies the
 * reference's rules on the device -- accept the longest prefix whose argmax
 * equals the draft (stopping after an accepted EOS), emit the correction or
 * the bonus token, move the cache position (the rewind), re-align the draft
 * pointer on the last emitted token within 40 drafts, the stuck guard (8
 * rounds), the chunk size 8 -> +4 up to 16 (2 after a boundary miss) -- and
 * writes the next round's ids, cache slot and k, or ends the loop when an EOS
 * was emitted, max_new_tokens are out, the draft is used up or k would be 0.
 * The host reads the emitted ids once, after the loop; the single-step
 * fallback decode that follows an exhausted draft stays with the caller
 * (speculative.py:541-560).
 *
 * verify: HOST array of max_chunk states, verify[k-1] for k + 1 tokens
 * (batch 1, m = k + 1, mode SB_MODE_VERIFY), all sharing one ids buffer
 * (>= max_chunk + 1), one ctrl block and one out_ids buffer.  spec: device
 * int32 [SB_SPEC_WORDS]: the host writes N_DRAFT, MAX_NEW, PROMPT and
 * MAX_ROUNDS before each launch, the loop writes the rest.  emitted: device
 * int64 [emit_capacity], emitted[0] = the prefill's token on entry.  The loop
 * never runs more than MAX_ROUNDS verify forwards (SB_SPEC_ERR = 1 if it
 * stopped there).  No reference counterpart for the graph itself (the
 * reference syncs with the host after every verify). */
#define SB_SPEC_N_EMIT 0     /* ids in emitted[] */
#define SB_SPEC_CACHE_POS 1  /* cache position after the last accepted token */
#define SB_SPEC_DRAFT_POS 2
#define SB_SPEC_CHUNK 3      /* current chunk size */
#define SB_SPEC_STUCK 4
#define SB_SPEC_ACCEPTED 5   /* accepted draft tokens (incl. re-alignments) */
#define SB_SPEC_VERIFIES 6   /* verify forwards run */
#define SB_SPEC_STOPPED 7    /* 1: an EOS was emitted */
#define SB_SPEC_ROUNDS 8
#define SB_SPEC_K 9          /* draft tokens in the round in flight */
#define SB_SPEC_ERR 10       /* 1: MAX_ROUNDS reached */
#define SB_SPEC_N_DRAFT 11   /* in */
#define SB_SPEC_MAX_NEW 12   /* in */
#define SB_SPEC_PROMPT 13    /* in: cache position of the first verify */
#define SB_SPEC_MAX_ROUNDS 14 /* in */
#define SB_SPEC_WORDS 16

typedef struct SbSpecLoop {
  const SbState* verify; /* HOST array [max_chunk] */
  int32_t max_chunk;
  int32_t draft_capacity;
  int32_t emit_capacity;
  int32_t _pad;
  int64_t eos_id;
  int32_t* spec;         /* [SB_SPEC_WORDS] */
  int64_t* emitted;      /* [emit_capacity] */
  const int64_t* draft;  /* [draft_capacity] */
} SbSpecLoop;

/* build and instantiate the loop's graph (captures every verify forward on
 * an internal stream); *loop_out receives an opaque handle */
int sb_spec_loop_create(const SbModel* model, const SbSpecLoop* loop, void** loop_out);
/* run the loop once on `stream` (asynchronous) */
int sb_spec_loop_launch(void* loop, sb_stream_t stream);
void sb_spec_loop_destroy(void* loop);

/* ---- prefill --------------------------------------------------------------
 * Prefill of `batch` right-padded prompts of T positions each, the eager
 * GraniteModel forward of LLMMega.prefill / BatchedLLMMega.prefill
 * (llm_mega.py:176-202, batched.py:222-276) on the library's kernels: per
 * layer q/k/v (RMSNorm prologue, RoPE at positions 0..T-1, K/V written to
 * cache slots 0..T-1 of streams 0..batch-1), causal attention over each
 * stream's keys [0, prompt_len[b]), o + residual, gate/up (RMSNorm, SwiGLU),
 * down + residual.  Rows of padding positions (>= prompt_len[b]) are not
 * computed where a whole 128-row token tile or 8-position query block is
 * padding; their hidden rows and cache slots hold unspecified values.  hidden [batch*T, hidden] bf16 holds the input embeddings
 * times the embedding multiplier on entry and the last layer's output rows on
 * exit (the caller applies the final norm / lm_head to the rows it needs).
 * T must be a multiple of 8 and <= max_len (pad the prompts; prompt_len
 * masks the padding); prompt_len: device int32 [batch], or NULL = T for all.
 * Scratch: q and attn [batch*T, n_q*128], act [sb_prefill_block_rows(), inter],
 * workspace of sb_prefill_workspace_bytes().  Every projection must be served
 * by the tensor-core GEMM (tile copies present; > 64 rows per block for
 * NVFP4 / INT8), else SB_ERR_CONFIG. */
size_t sb_prefill_workspace_bytes(const SbModel* model, int32_t batch, int32_t T);
int32_t sb_prefill_block_rows(const SbModel* model, int32_t batch, int32_t T);
int sb_prefill(const SbModel* model, uint16_t* hidden, int32_t batch, int32_t T, const int32_t* prompt_len,
               uint16_t* q, uint16_t* attn, uint16_t* act, void* workspace, size_t workspace_bytes,
               sb_stream_t stream);

/* ---- single ops (each one replaces one reference call site) ------------- */
/* y[m, :] = x[m, :] W^T, bf16 out: nn.Linear (llm_mega.py:534-536,560,572-573,579,588).
 * Any m >= 1; y columns in packed row order.
 * GEMV kernels only (no workspace). */
int sb_linear(const SbLinear* lin, const uint16_t* x, uint16_t* y, int32_t m, int32_t use_pdl,
              sb_stream_t stream);
/* bytes of workspace sb_linear_ex needs to run (lin, m) on the tensor-core
 * GEMM (0: that path does not serve it) */
size_t sb_linear_workspace_bytes(const SbLinear* lin, int32_t m);
/* sb_linear with operand scratch: with lin->w_tc set and m > 8 the rows go
 * through the tcgen05 GEMM (token tiles of 128 in one launch, blocks of up to
 * 8192 rows; prefill projections) */
int sb_linear_ex(const SbLinear* lin, const uint16_t* x, uint16_t* y, int32_t m, void* workspace,
                 size_t workspace_bytes, int32_t use_pdl, sb_stream_t stream);
/* exact dequantisation of a packed layer to fp32 [n, k] (rows in packed order,
 * padding rows dropped); the quantised formats have no reference counterpart */
int sb_dequant_f32(const SbLinear* lin, float* out, sb_stream_t stream);
/* same, rounded to bf16 (used for prefill GEMMs) */
int sb_dequant_bf16(const SbLinear* lin, uint16_t* out, sb_stream_t stream);
/* fused_rmsnorm (llm_kernels.py:124-139) */
int sb_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int32_t rows, int32_t n, float eps,
               sb_stream_t stream);
/* fused_silu_mul (llm_kernels.py:267-285) */
int sb_silu_mul(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t count, sb_stream_t stream);
/* fused_residual_scale (llm_kernels.py:320-336) */
int sb_residual_scale(const uint16_t* x, const uint16_t* y, uint16_t* z, int64_t count, float alpha,
                      sb_stream_t stream);
/* RoPE of (llm_mega.py:539-543): x [rows, 128] bf16 in place, row r at position pos[r / heads] */
int sb_rope(uint16_t* x, int32_t rows, int32_t heads, const int32_t* pos, const uint16_t* cos_tab,
            const uint16_t* sin_tab, sb_stream_t stream);
/* argmax over bf16 rows, lowest index on ties (torch semantics): static_logits.argmax(-1) */
int sb_argmax_bf16(const uint16_t* x, int32_t rows, int32_t n, int64_t* out, sb_stream_t stream);
/* decode attention for one layer (llm_mega.py:546-556 incl. StaticLayer.update and
 * repeat_kv): q [B*m, n_q*128], caches as SbLayer, out [B*m, n_q*128] */
int sb_attention(const SbModel* model, const SbState* state, int32_t layer, sb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* STARLING_B200_H */
