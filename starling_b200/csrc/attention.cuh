// Decode / verify attention over the static KV cache.  See attention.cu.
#pragma once
#include "common.cuh"

namespace sb {

struct AttnParams {
  const uint16_t* q;        // [B*m_per][n_q*128]
  const uint16_t* k_cache;  // [max_batch][n_kv][max_len][128]
  const uint16_t* v_cache;
  uint16_t* out;  // [B*m_per][n_q*128]
  int n_q, n_kv, max_len, m_per;
  float attn_mult;
  int32_t* ctrl;              // SB_CTRL_SLOT, SB_CTRL_PADLEN (read), SB_CTRL_ERR (written on a failed wait)
  const int32_t* prompt_len;  // [B] or nullptr
  int split;                  // CTAs per (stream, KV head), one cluster
  int chunk_cap;              // keys per CTA at most: attn_key_capacity(max_len, split)
  int slots;                  // ring slots of 64 keys (K or V)
  long long cache_rows;       // max_batch * n_kv * max_len (rows of 128 of each cache)
  int qblocks;                // query blocks of m_per tokens per stream: block qb has its tokens
                              // at cache slots ctrl[SLOT] + qb * m_per + (0..m_per-1) (prefill); 1 otherwise
  // When opnd is set (qblocks == 1), the output rows are also written as the
  // o-projection GEMM's activation operand (one token tile, gemm_tc.cu's
  // layout): bf16 rows, or (opnd_fp8) two e4m3 terms per element with one
  // power-of-two shift per (KV head, token) -- the o GEMM splits K over n_kv
  // ranks, one KV head's n_q / n_kv heads each -- in opnd_shift[kvh][opnd_mp].
  uint8_t* opnd;
  int32_t* opnd_shift;
  int opnd_mp, opnd_np, opnd_fp8;
};

int attn_tile_keys(int split);
int attn_key_capacity(int max_len, int split);
size_t attn_smem_bytes(int R, int chunk_cap, int slots, int tk);
int attn_launch(const AttnParams& p, int batch, bool pdl, cudaStream_t stream);
// Prefill (attention_pf.cu): causal attention of T prompt positions per stream
// (queries p.q / p.out rows b * T + pos, keys cache slots 0..pos), 128 query
// rows per CTA; uses p.q, k_cache, v_cache, out, n_q, n_kv, max_len,
// attn_mult, prompt_len.
bool attn_prefill_ok(int n_q, int n_kv);
int attn_prefill_launch(const AttnParams& p, int batch, int T, cudaStream_t stream);

}  // namespace sb
