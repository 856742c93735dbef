// Row-owned epilogues of the tensor-core GEMM (gemm_tc.cu).
//
// The lanes of a warp hold consecutive packed rows (lane = row within a group
// of 32), so the two rows of a RoPE pair or of a gate/up pair sit in adjacent
// lanes and meet through one shuffle.  Each call covers one row per lane and
// CNT consecutive tokens [m0, m0 + CNT), the values in registers: stores are
// coalesced over the lanes and every global load of a call (residual rows,
// RoPE tables) is in flight at once.  Same operations and rounding points as
// gemv_epilogue (gemv_epi.cuh).
#pragma once
#include "gemv.cuh"
#include "operand.cuh"

namespace sb {

// v[i]: dot product of this lane's row and token m0 + i, activation scaling
// undone, weight scale not yet applied.  row_ok: the row exists (row < n).
// tok0: first token of the token tile (token m0 + i of the call is row
// tok0 + m0 + i of the outputs; argmax needs tok0 = 0).
// Must be called by full warps with warp-uniform m0.  ARGMAX keeps a running
// best per (warp, token) in wb_val/wb_idx[warp * 128 + m].
// EPI: the epilogue (EPI_*), fixed at compile time.
// QKV: tokpos (shared memory) describes token m0 + i of the call (the token
// tile starting at tok0): [m0 + i] its RoPE position, [129 + m0 + i] its
// stream, [257 + m0 + i] its position in the stream, [128] the cache slot of
// position 0; nullptr: compute them from the control block and rope_off here.
template <int FMT, int CNT, int EPI>
__device__ __forceinline__ void tc_epi(const GemvParams& p, int row, bool row_ok, float* v, int m0, int M,
                                       float* wb_val, int* wb_idx, int warp, int tok0,
                                       const int* tokpos = nullptr) {
  const int lane = threadIdx.x & 31;
  float rs = 1.f;
  if (row_ok) {
    if (FMT == SB_FMT_FP8 || FMT == SB_FMT_INT8) rs = reinterpret_cast<const float*>(p.scale)[row];
    if (FMT == SB_FMT_NVFP4) rs = p.gscale;
  }
#pragma unroll
  for (int i = 0; i < CNT; ++i) v[i] *= rs;
  if constexpr (EPI == EPI_STORE) {
#pragma unroll
    for (int i = 0; i < CNT; ++i)
      if (row_ok && m0 + i < M) p.y[static_cast<size_t>(tok0 + m0 + i) * p.n + row] = f_to_bf16_bits(v[i]);
  } else if constexpr (EPI == EPI_RESID) {
    // hidden = hidden + bf16(res_mult * bf16(y))   (llm_kernels.py:306-313)
    float h[CNT];
#pragma unroll
    for (int i = 0; i < CNT; ++i)
      h[i] = (row_ok && m0 + i < M) ? u16_to_f(p.y[static_cast<size_t>(tok0 + m0 + i) * p.n + row]) : 0.f;
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
      const bool ok = row_ok && m0 + i < M;
      v[i] = ok ? bf(h[i] + bf(p.res_mult * bf(v[i]))) : 0.f;  // the new hidden value (decode chain)
      if (ok) p.y[static_cast<size_t>(tok0 + m0 + i) * p.n + row] = f_to_bf16_bits(v[i]);
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // act = bf16(bf16(silu(gate)) * up) (llm_kernels.py:252-260); gate row 2i, up row 2i+1
    const int inter = p.n / 2;
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
      const float up = __shfl_down_sync(0xffffffffu, v[i], 1);
      float act = 0.f;
      if (row_ok && !(row & 1) && m0 + i < M) {
        const float gv = bf(v[i]);
        const float sg = bf(gv / (1.f + expf(-gv)));
        act = bf(sg * bf(up));
        p.y[static_cast<size_t>(tok0 + m0 + i) * inter + row / 2] = f_to_bf16_bits(act);
      }
      v[i] = act;  // even lanes: the activation (for the next operand), odd lanes 0
    }
  } else if constexpr (EPI == EPI_QKV) {
    // q/k: RoPE with each product rounded to bf16 (llm_mega.py:539-543); k/v to
    // cache slot ctrl[SLOT] + token (StaticLayer.update, cache_utils.py:308-335)
    const int qk_rows = (p.n_q + p.n_kv) * 128;
    const int slot_base = tokpos ? tokpos[128] : p.ctrl[SB_CTRL_SLOT];
    const int head = row >> 7, within = row & 127;
    const bool odd = within & 1;
    const int j = within >> 1;
    const bool is_qk = row < qk_rows;  // warp-uniform: 32-row groups never straddle 128-row heads
    float cs[CNT], sn[CNT];
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
      cs[i] = 0.f;
      sn[i] = 0.f;
      if (is_qk && row_ok && m0 + i < M) {
        int pos;
        if (tokpos) {
          pos = tokpos[m0 + i];
        } else {
          const int m = tok0 + m0 + i, b = m / p.m_per, mi = m % p.m_per;
          pos = slot_base + mi - (p.rope_off ? p.rope_off[b] : 0);
          pos = pos < 0 ? 0 : (pos >= p.rope_max ? p.rope_max - 1 : pos);
        }
        cs[i] = u16_to_f(p.cos_tab[pos * 64 + j]);
        sn[i] = u16_to_f(p.sin_tab[pos * 64 + j]);
      }
    }
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
      const float other = __shfl_xor_sync(0xffffffffu, v[i], 1);
      if (!row_ok || m0 + i >= M) continue;
      const int m = tok0 + m0 + i;
      const int b = tokpos ? tokpos[129 + m0 + i] : m / p.m_per, mi = tokpos ? tokpos[257 + m0 + i] : m % p.m_per;
      const int slot = slot_base + mi;
      const bool slot_ok = slot >= 0 && slot < p.max_len;
      if (is_qk) {
        const float mine = bf(v[i]), oth = bf(other);
        // even row: x1 (dim j) -> x1 cos - x2 sin ; odd row: x2 (dim j+64) -> x2 cos + x1 sin
        const float o = odd ? bf(mine * cs[i]) + bf(oth * sn[i]) : bf(mine * cs[i]) - bf(oth * sn[i]);
        const int dim = odd ? j + 64 : j;
        if (head < p.n_q) {
          p.q_out[static_cast<size_t>(m) * p.n_q * 128 + head * 128 + dim] = f_to_bf16_bits(o);
        } else if (slot_ok) {
          p.k_cache[((static_cast<size_t>(b) * p.n_kv + (head - p.n_q)) * p.max_len + slot) * 128 + dim] =
              f_to_bf16_bits(o);
        }
      } else if (slot_ok) {
        p.v_cache[((static_cast<size_t>(b) * p.n_kv + (head - p.n_q - p.n_kv)) * p.max_len + slot) * 128 + within] =
            f_to_bf16_bits(v[i]);
      }
    }
  } else if constexpr (EPI == EPI_ARGMAX) {
    // logits = bf16(bf16(y) * (1/logits_scaling)); running (value, index) best per (warp, token)
#pragma unroll
    for (int i = 0; i < CNT; ++i) {
      const int m = m0 + i;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      if (row_ok && m < M) {
        const float lv = bf(bf(v[i]) * p.logits_mult);
        if (p.logits) p.logits[static_cast<size_t>(m) * p.n + row] = f_to_bf16_bits(lv);
        bv = lv;
        bi = row;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (am_better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0 && m < M) {
        float* pv = wb_val + warp * 128 + m;
        int* pi = wb_idx + warp * 128 + m;
        if (am_better(bv, bi, *pv, *pi)) {
          *pv = bv;
          *pi = bi;
        }
      }
    }
  }
}

}  // namespace sb
