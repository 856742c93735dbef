// Epilogues of the persistent decode GEMV (gemv_dec.cu): the same fused
// operations as k_gemv's (gemv.cu), applied to a block of reduced rows.
#pragma once
#include "gemv.cuh"

namespace sb {

// tot[lrow * M + m] holds the reduced, activation-unscaled dot product of
// packed row row0 + lrow and token m.  first/last mark the CTA's first and
// last block (argmax keeps a running best per token across blocks).  Run by
// the nthr (a multiple of 32) threads tid = 0..nthr-1 of the block; it has no
// barrier inside.
// EPIC >= 0 fixes the epilogue at compile time (only that branch is
// generated); -1 dispatches on p.epi.
template <int FMT, int EPIC = -1>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, const float* tot, int row0, int nrow, int M,
                                              int* s_best, float* s_bval, bool first, bool last, int tid, int nthr) {
  const int lane = tid & 31, warp = tid >> 5, W = nthr >> 5;
  const int epi = EPIC >= 0 ? EPIC : p.epi;
  auto fin = [&](int lrow, int m) -> float {
    float v = tot[lrow * M + m];
    if (FMT == SB_FMT_NVFP4) v *= p.gscale;
    if (FMT == SB_FMT_FP8 || FMT == SB_FMT_INT8) v *= reinterpret_cast<const float*>(p.scale)[row0 + lrow];
    return v;
  };
  if (epi == EPI_STORE) {
    for (int i = tid; i < nrow * M; i += nthr) {
      const int m = i / nrow, lrow = i % nrow, row = row0 + lrow;
      if (row < p.n) p.y[static_cast<size_t>(m) * p.n + row] = f_to_bf16_bits(fin(lrow, m));
    }
  } else if (epi == EPI_RESID) {
    // hidden = hidden + bf16(res_mult * bf16(y))   (llm_kernels.py:306-313)
    for (int i = tid; i < nrow * M; i += nthr) {
      const int m = i / nrow, lrow = i % nrow, row = row0 + lrow;
      if (row < p.n) {
        uint16_t* hp = p.y + static_cast<size_t>(m) * p.n + row;
        uint16_t* cp = p.resid_cache ? p.resid_cache + m * p.rc_stride + (row - p.rc_row0) : nullptr;
        const uint16_t nv = f_to_bf16_bits(u16_to_f(cp ? *cp : __ldcg(hp)) + bf(p.res_mult * bf(fin(lrow, m))));
        *hp = nv;
        if (cp) *cp = nv;
      }
    }
  } else if (epi == EPI_SWIGLU) {
    // act = bf16(bf16(silu(gate)) * up)   (llm_kernels.py:252-260); rows interleave gate/up
    const int inter = p.n / 2, np = nrow / 2;
    for (int i = tid; i < np * M; i += nthr) {
      const int m = i / np, lp = i % np, lrow = 2 * lp, row = row0 + lrow;
      if (row < p.n) {
        const float gv = bf(fin(lrow, m));
        const float uv = bf(fin(lrow + 1, m));
        const float sg = bf(gv / (1.f + expf(-gv)));
        p.y[static_cast<size_t>(m) * inter + row / 2] = f_to_bf16_bits(sg * uv);
      }
    }
  } else if (epi == EPI_QKV) {
    // q/k: RoPE with each product rounded to bf16 (llm_mega.py:539-543); k/v
    // to cache slot ctrl[SLOT] + token (StaticLayer.update, cache_utils.py:308-335)
    const int qk_rows = (p.n_q + p.n_kv) * 128;
    const int slot_base = p.ctrl[SB_CTRL_SLOT];
    for (int i = tid; i < nrow * M; i += nthr) {
      const int m = i / nrow, lrow = i % nrow, row = row0 + lrow;
      if (row >= p.n) continue;
      const int b = m / p.m_per, mi = m % p.m_per;
      const int slot = slot_base + mi;
      const bool slot_ok = slot >= 0 && slot < p.max_len;
      const int head = row >> 7, within = row & 127;
      if (row < qk_rows) {
        if (within & 1) continue;
        const int j = within >> 1;
        int pos = slot - (p.rope_off ? p.rope_off[b] : 0);
        pos = pos < 0 ? 0 : (pos >= p.rope_max ? p.rope_max - 1 : pos);
        const float x1 = bf(fin(lrow, m));
        const float x2 = bf(fin(lrow + 1, m));
        const float cs = u16_to_f(p.rope_cache ? p.rope_cache[m * 128 + j] : p.cos_tab[pos * 64 + j]);
        const float sn = u16_to_f(p.rope_cache ? p.rope_cache[m * 128 + 64 + j] : p.sin_tab[pos * 64 + j]);
        const uint16_t o1 = f_to_bf16_bits(bf(x1 * cs) - bf(x2 * sn));
        const uint16_t o2 = f_to_bf16_bits(bf(x2 * cs) + bf(x1 * sn));
        if (head < p.n_q) {
          uint16_t* qo = p.q_out + static_cast<size_t>(m) * p.n_q * 128 + head * 128;
          qo[j] = o1;
          qo[j + 64] = o2;
        } else if (slot_ok) {
          uint16_t* kc = p.k_cache + ((static_cast<size_t>(b) * p.n_kv + (head - p.n_q)) * p.max_len + slot) * 128;
          kc[j] = o1;
          kc[j + 64] = o2;
        }
      } else if (slot_ok) {
        p.v_cache[((static_cast<size_t>(b) * p.n_kv + (head - p.n_q - p.n_kv)) * p.max_len + slot) * 128 + within] =
            f_to_bf16_bits(fin(lrow, m));
      }
    }
  } else if (epi == EPI_ARGMAX) {
    // logits = bf16(bf16(y) * (1/logits_scaling)); running (value, index) best
    for (int m = warp; m < M; m += W) {
      float bv = first ? -INFINITY : s_bval[m];
      int bi = first ? 0x7fffffff : s_best[m];
      for (int lrow = lane; lrow < nrow; lrow += 32) {
        const int row = row0 + lrow;
        if (row >= p.n) continue;
        const float lv = bf(bf(fin(lrow, m)) * p.logits_mult);
        if (p.logits) p.logits[static_cast<size_t>(m) * p.n + row] = f_to_bf16_bits(lv);
        if (am_better(lv, row, bv, bi)) {
          bv = lv;
          bi = row;
        }
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
      if (lane == 0) {
        s_bval[m] = bv;
        s_best[m] = bi;
      }
    }
  }
  (void)last;
}

// Argmax tail: publish this CTA's best per token, and in the last CTA to
// arrive reduce all partials (total order on (value desc, index asc), so the
// result is deterministic) and apply the decode / verify feedback.
__device__ __forceinline__ void gemv_argmax_finish(const GemvParams& p, int* s_best, float* s_bval, int M,
                                                   bool has_rows, int* s_flag) {
  if (p.epi != EPI_ARGMAX) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, W = blockDim.x >> 5;
  const int cta = blockIdx.x;
  if (tid < M) {
    p.part_val[static_cast<size_t>(cta) * M + tid] = has_rows ? s_bval[tid] : -INFINITY;
    p.part_idx[static_cast<size_t>(cta) * M + tid] = has_rows ? s_best[tid] : 0x7fffffff;
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const int prev = atomicAdd(p.counter, 1);
    *s_flag = prev == p.n_ctas - 1;
  }
  __syncthreads();
  if (!*s_flag) return;
  __threadfence();
  // a warp per token; each lane's partials are all loaded before any is
  // compared (one L2 round trip instead of one per 32 CTAs).  The order is
  // total, so the result does not depend on the comparison order.
  constexpr int kPerLane = 12;  // up to 384 CTAs in registers; more take a second loop
  for (int m = warp; m < M; m += W) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    float vv[kPerLane];
    int iv[kPerLane];
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int q = lane + 32 * j;
      vv[j] = q < p.n_ctas ? __ldcg(p.part_val + static_cast<size_t>(q) * M + m) : -INFINITY;
      iv[j] = q < p.n_ctas ? __ldcg(p.part_idx + static_cast<size_t>(q) * M + m) : 0x7fffffff;
    }
#pragma unroll
    for (int j = 0; j < kPerLane; ++j)
      if (am_better(vv[j], iv[j], bv, bi)) {
        bv = vv[j];
        bi = iv[j];
      }
    for (int q = lane + 32 * kPerLane; q < p.n_ctas; q += 32) {
      const float v = __ldcg(p.part_val + static_cast<size_t>(q) * M + m);
      const int ix = __ldcg(p.part_idx + static_cast<size_t>(q) * M + m);
      if (am_better(v, ix, bv, bi)) {
        bv = v;
        bi = ix;
      }
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
    if (lane == 0) s_best[m] = bi;
  }
  __syncthreads();
  if (p.mode == SB_MODE_VERIFY) {
    if (tid < M && p.out_ids) p.out_ids[tid] = s_best[tid];
    if (tid == 0) {
      int j = 0;
      while (j < M - 1 && static_cast<int64_t>(s_best[j]) == p.ids_io[j + 1]) ++j;
      p.ctrl[SB_CTRL_ACCEPT] = j;
    }
  } else {
    for (int b = tid; b < M; b += blockDim.x) {
      const int64_t tok = s_best[b];
      int64_t out = tok, next = tok;
      if (p.finished) {
        if (p.finished[b]) {
          out = p.pad_id;
          next = p.pad_id;
        } else if (tok == p.eos_id) {
          p.finished[b] = 1;
          next = p.pad_id;
        }
      }
      if (p.out_ids) p.out_ids[static_cast<size_t>(p.step) * p.batch + b] = out;
      p.ids_io[b] = next;
    }
    if (tid == 0 && p.mode == SB_MODE_DECODE) p.ctrl[SB_CTRL_SLOT] += 1;
  }
  if (tid == 0) *p.counter = 0;
}

}  // namespace sb
