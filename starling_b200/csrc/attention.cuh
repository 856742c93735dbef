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
  const int32_t* ctrl;        // SB_CTRL_SLOT, SB_CTRL_PADLEN
  const int32_t* prompt_len;  // [B] or nullptr
  int split;                  // CTAs per cluster splitting the keys
  int chunk_cap;              // ceil(max_len / split)
};

size_t attn_smem_bytes(int R, int chunk_cap);
int attn_launch(const AttnParams& p, int batch, bool pdl, cudaStream_t stream);

}  // namespace sb
