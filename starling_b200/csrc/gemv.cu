// Weight-only dequant-GEMV for decode (m <= 64 token rows), sm_100a.
//
// Replaces the nn.Linear calls of the reference decode step
// (src/starling/granite/llm_mega.py:534-536,560,572-573,579,588) together
// with the glue around them: the RMSNorm before q/k/v and gate/up
// (llm_kernels.py:93-139), RoPE + the StaticCache write after q/k/v
// (llm_mega.py:538-546), SiLU*mul after gate/up (llm_kernels.py:241-285), the
// residual scale-add after o and down (llm_kernels.py:295-336) and the
// lm_head logit scaling + greedy argmax + token feedback
// (llm_mega.py:588-589, multistep.py:181-188).
//
// Design (B=1 decode is HBM-bound weight streaming):
//  * weights are pre-packed so that each lane's 16-byte load is exactly its
//    mma.m16n8k16 A-fragment for one "kgroup" of K (64 nvfp4 / 32 fp8,int8 /
//    16 bf16 elements); a warp load is 512 contiguous bytes;
//  * low-precision weights are decoded in registers to f16 (nvfp4: e2m1 code
//    times its e4m3 block scale, an exact f16 product; fp8/int8: exact) and
//    multiplied on the tensor cores against the activation rows held in
//    shared memory (f16, scaled by a power of two chosen per row so the
//    conversion from bf16 is exact); the fp32 per-tensor / per-row scale and
//    the power of two are applied once per output;
//  * each CTA owns `rt` 16-row tiles; its warps split the CTA's K range and
//    reduce through shared memory in a fixed order; when K is split across
//    the `ck` CTAs of a thread-block cluster the partial sums are reduced
//    through distributed shared memory, again in a fixed order, so results
//    are deterministic;
//  * before waiting on the previous kernel (programmatic dependent launch)
//    every CTA bulk-prefetches its weight bytes into L2, so weight streaming
//    of layer i+1 overlaps the tail of layer i.
#include <cooperative_groups.h>

#include "gemv.cuh"

namespace cg = cooperative_groups;

namespace sb {

int kgroup_elems(int fmt) { return fmt == SB_FMT_NVFP4 ? 64 : (fmt == SB_FMT_BF16 ? 16 : 32); }

template <int FMT, int NT>
__device__ __forceinline__ void mma_rows(float (&acc)[NT][4], const uint32_t* A, const uint16_t* xs,
                                         int xs_stride, int kk, int M, int g, int c) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    int n = nt * 8 + g;
    n = n < M ? n : M - 1;
    const uint16_t* xr = xs + n * xs_stride + kk + 2 * c;
    const uint32_t b0 = *reinterpret_cast<const uint32_t*>(xr);
    const uint32_t b1 = *reinterpret_cast<const uint32_t*>(xr + 8);
    if constexpr (FMT == SB_FMT_BF16)
      mma_bf16(acc[nt], A, b0, b1);
    else
      mma_f16(acc[nt], A, b0, b1);
  }
}

template <int FMT, int NT>
__device__ __forceinline__ void process_kgroup(const uint4 a, const uint2 s, int kbase, const uint16_t* xs,
                                               int xs_stride, int M, int g, int c, float (&acc)[NT][4]) {
  if constexpr (FMT == SB_FMT_NVFP4) {
    const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t A[4];
      A[0] = e2m1x2_to_h2(wv[ks]);
      A[1] = e2m1x2_to_h2(wv[ks] >> 8);
      A[2] = e2m1x2_to_h2(wv[ks] >> 16);
      A[3] = e2m1x2_to_h2(wv[ks] >> 24);
      const uint32_t sp = ((ks < 2) ? s.x : s.y) >> ((ks & 1) * 16);
      const uint32_t sh = e4m3x2_to_h2(sp);  // {scale of row g, scale of row g+8}
      const uint32_t slo = __byte_perm(sh, 0, 0x1010);
      const uint32_t shi = __byte_perm(sh, 0, 0x3232);
      A[0] = hmul2_u32(A[0], slo);
      A[2] = hmul2_u32(A[2], slo);
      A[1] = hmul2_u32(A[1], shi);
      A[3] = hmul2_u32(A[3], shi);
      mma_rows<FMT, NT>(acc, A, xs, xs_stride, kbase + ks * 16, M, g, c);
    }
  } else if constexpr (FMT == SB_FMT_FP8) {
    const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t A[4];
      A[0] = e4m3x2_to_h2(wv[2 * ks]);
      A[1] = e4m3x2_to_h2(wv[2 * ks] >> 16);
      A[2] = e4m3x2_to_h2(wv[2 * ks + 1]);
      A[3] = e4m3x2_to_h2(wv[2 * ks + 1] >> 16);
      mma_rows<FMT, NT>(acc, A, xs, xs_stride, kbase + ks * 16, M, g, c);
    }
  } else if constexpr (FMT == SB_FMT_INT8) {
    const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      uint32_t A[4];
      i8x4_to_h2x2(wv[2 * ks], A[0], A[1]);
      i8x4_to_h2x2(wv[2 * ks + 1], A[2], A[3]);
      mma_rows<FMT, NT>(acc, A, xs, xs_stride, kbase + ks * 16, M, g, c);
    }
  } else {
    const uint32_t A[4] = {a.x, a.y, a.z, a.w};
    mma_rows<FMT, NT>(acc, A, xs, xs_stride, kbase, M, g, c);
  }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(512) k_gemv(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int KGE = KG<FMT>::E;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, W = blockDim.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int ck = p.ck;
  const int rank = ck > 1 ? static_cast<int>(cg::this_cluster().block_rank()) : 0;
  const int cluster_id = blockIdx.x / ck;
  const int tile0 = cluster_id * p.rt;
  const int k_cta = p.k / ck;
  const int k0 = rank * k_cta;
  const int kg_cta = k_cta / KGE;
  const int kg0 = k0 / KGE;
  // plain row blocks (EPI_STORE only): gridDim.y chunks of up to 64 rows
  const int M = gridDim.y > 1 ? min(64, p.m - static_cast<int>(blockIdx.y) * 64) : p.m;
  const size_t row_off = static_cast<size_t>(blockIdx.y) * 64;
  const uint16_t* const xin = p.x ? p.x + row_off * p.k : nullptr;
  uint16_t* const yout = p.y ? p.y + row_off * p.n : nullptr;
  const int ntile = min(p.rt, p.n_tiles - tile0);
  const int rt16 = p.rt * 16;
  // Each warp owns one row tile; the wpt warps of a tile split its K range
  // (kgroups my_sub, my_sub + wpt, ...).
  const int wpt = W / p.rt;
  const int my_tile = warp / wpt, my_sub = warp % wpt;
  const bool tile_live = my_tile < ntile;
  const size_t tt = static_cast<size_t>(tile0 + (tile_live ? my_tile : 0));
  const uint4* wt = reinterpret_cast<const uint4*>(p.w) + (tt * p.kg_total + kg0) * 32 + lane;
  const uint2* st = reinterpret_cast<const uint2*>(p.scale) + (tt * p.kg_total + kg0) * 8 + g;

  // ---- 1. weights do not depend on the previous kernel: start streaming them
  //         before waiting for it (first PRE kgroups per warp into registers,
  //         the rest of the CTA's range into L2) ---------------------------------
  constexpr int PRE = 8;
  uint4 a[PRE];
  uint2 s[PRE];
#pragma unroll
  for (int u = 0; u < PRE; ++u) {
    const int kg = my_sub + u * wpt;
    if (tile_live && kg < kg_cta) {
      a[u] = ldg_stream(wt + static_cast<size_t>(kg) * 32);
      if constexpr (FMT == SB_FMT_NVFP4) s[u] = ldg_stream2(st + static_cast<size_t>(kg) * 8);
    }
  }
  if (tid == 0 && kg_cta > PRE * wpt) {
    const int kg_rest = PRE * wpt;
    for (int r = 0; r < ntile; ++r) {
      const size_t t = static_cast<size_t>(tile0 + r);
      prefetch_l2(p.w + (t * p.kg_total + kg0 + kg_rest) * 512, static_cast<uint32_t>(kg_cta - kg_rest) * 512u);
      if (FMT == SB_FMT_NVFP4)
        prefetch_l2(p.scale + (t * p.kg_total + kg0 + kg_rest) * 64, static_cast<uint32_t>(kg_cta - kg_rest) * 64u);
    }
  }
  pdl_wait();
  pdl_launch();

  // ---- 2. shared memory --------------------------------------------------------
  const int xs_stride = k_cta + 8;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  size_t off = (static_cast<size_t>(M) * xs_stride * 2 + 15) & ~size_t(15);
  float* red = reinterpret_cast<float*>(smem + off);        // [W][16][M]
  float* tot = red + static_cast<size_t>(W) * 16 * M;       // [rt16][M]
  int* xshift = reinterpret_cast<int*>(tot + rt16 * M);     // [64]
  int* s_best = xshift + 64;                                // [64]
  float* s_bval = reinterpret_cast<float*>(s_best + 64);     // [64]
  int* s_flag = reinterpret_cast<int*>(s_bval + 64);        // [4]
  float* s_red = reinterpret_cast<float*>(s_flag + 4);      // [16] per-warp partial sums
  float* s_amx = s_red + 16;                                // [16] per-warp partial maxima

  // ---- 3. stage the activation rows (prologue) -----------------------------------
  // A row is handled by wpr = W / M warps (one pass when M <= W) whose loads
  // are all independent; per-row sums and maxima are combined through shared
  // memory in a fixed order.
  {
    const int wpr = W / M >= 1 ? W / M : 1;
    const int nslot = W / wpr;
    const int slot = warp / wpr, sub = warp % wpr;
    const int gt = sub * 32 + lane, gn = wpr * 32;
    const bool norm = p.pro != PRO_NONE;
    for (int m0 = 0; m0 < M; m0 += nslot) {
      const int m = m0 + slot;
      const bool live = slot < nslot && m < M;
      const uint16_t* src = xin;
      if (live) {
        if (p.pro == PRO_EMBED) {
          int64_t id = p.ids[m];
          id = id < 0 ? 0 : (id >= p.embed_rows ? p.embed_rows - 1 : id);  // never read outside the table
          src = p.embed + static_cast<size_t>(id) * p.k;
        } else {
          src = xin + static_cast<size_t>(m) * p.k;
        }
      }
      float rstd = 1.f;
      if (norm) {
        float ss = 0.f;
        if (live) {
          const bool write_h = p.pro == PRO_EMBED && blockIdx.x == 0 && p.hidden_out != nullptr;
#pragma unroll 4
          for (int k = gt * 8; k < p.k; k += gn * 8) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4*>(src + k), f);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              if (p.pro == PRO_EMBED) f[j] = bf(f[j] * p.emb_mult);  // embed_tokens(ids) * 12 (llm_mega.py:514)
              ss += f[j] * f[j];
            }
            if (write_h) *reinterpret_cast<uint4*>(p.hidden_out + static_cast<size_t>(m) * p.k + k) = pack8(f);
          }
        }
        ss = warp_sum(ss);
        if (lane == 0) s_red[warp] = ss;
        __syncthreads();
        if (live) {
          float tsum = 0.f;
          for (int q = 0; q < wpr; ++q) tsum += s_red[slot * wpr + q];
          rstd = 1.f / sqrtf(tsum / static_cast<float>(p.k) + p.eps);
        }
      }
      float amax = 0.f;
      if (live) {
#pragma unroll 4
        for (int k = gt * 8; k < k_cta; k += gn * 8) {
          float f[8];
          unpack8(*reinterpret_cast<const uint4*>(src + k0 + k), f);
          if (norm) {
            float w8[8];
            unpack8(*reinterpret_cast<const uint4*>(p.norm_w + k0 + k), w8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float h = p.pro == PRO_EMBED ? bf(f[j] * p.emb_mult) : f[j];
              f[j] = bf(w8[j] * bf(h * rstd));  // weight * bf16(x * rstd)  (modeling_granite.py:192-197)
            }
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
          *reinterpret_cast<uint4*>(xs + m * xs_stride + k) = pack8(f);
        }
      }
      if (FMT != SB_FMT_BF16) {
        amax = warp_max(amax);
        if (lane == 0) s_amx[warp] = amax;
        __syncthreads();
        if (live) {
          float am = 0.f;
          for (int q = 0; q < wpr; ++q) am = fmaxf(am, s_amx[slot * wpr + q]);
          int e = 0;
          if (am > 0.f) frexpf(am, &e);
          const int shift = 15 - e;  // row max * 2^shift in [2^14, 2^15): exact bf16 -> f16
          for (int k = gt * 8; k < k_cta; k += gn * 8) {  // same thread wrote these elements
            float f[8];
            unpack8(*reinterpret_cast<const uint4*>(xs + m * xs_stride + k), f);
            uint32_t h[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              __half2 hh = __floats2half2_rn(ldexpf(f[2 * j], shift), ldexpf(f[2 * j + 1], shift));
              h[j] = *reinterpret_cast<uint32_t*>(&hh);
            }
            *reinterpret_cast<uint4*>(xs + m * xs_stride + k) = make_uint4(h[0], h[1], h[2], h[3]);
          }
          if (sub == 0 && lane == 0) xshift[m] = shift;
        }
      } else if (live && sub == 0 && lane == 0) {
        xshift[m] = 0;
      }
      __syncthreads();  // xs rows complete; s_red / s_amx free for the next pass
    }
  }

  // ---- 4. the weight tile through the tensor cores ---------------------------------
  float acc[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
  for (int u = 0; u < PRE; ++u) {
    const int kg = my_sub + u * wpt;
    if (tile_live && kg < kg_cta) process_kgroup<FMT, NT>(a[u], s[u], kg * KGE, xs, xs_stride, M, g, c, acc);
  }
  for (int base = PRE; my_sub + base * wpt < kg_cta; base += PRE) {  // ranges longer than the preload
#pragma unroll
    for (int u = 0; u < PRE; ++u) {
      const int kg = my_sub + (base + u) * wpt;
      if (tile_live && kg < kg_cta) {
        a[u] = ldg_stream(wt + static_cast<size_t>(kg) * 32);
        if constexpr (FMT == SB_FMT_NVFP4) s[u] = ldg_stream2(st + static_cast<size_t>(kg) * 8);
      }
    }
#pragma unroll
    for (int u = 0; u < PRE; ++u) {
      const int kg = my_sub + (base + u) * wpt;
      if (tile_live && kg < kg_cta) process_kgroup<FMT, NT>(a[u], s[u], kg * KGE, xs, xs_stride, M, g, c, acc);
    }
  }
  {
    float* rw = red + static_cast<size_t>(warp) * 16 * M;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int col = nt * 8 + 2 * c;
      if (col < M) {
        rw[g * M + col] = acc[nt][0];
        rw[(g + 8) * M + col] = acc[nt][2];
      }
      if (col + 1 < M) {
        rw[g * M + col + 1] = acc[nt][1];
        rw[(g + 8) * M + col + 1] = acc[nt][3];
      }
    }
  }
  __syncthreads();

  // ---- 5. reduce: the tile's warps (fixed order), then cluster ranks (fixed order)
  const int nrow = ntile * 16;
  for (int i = tid; i < nrow * M; i += blockDim.x) {
    const int lrow = i / M, m = i % M;
    const int r = lrow >> 4, rr = lrow & 15;
    float sum = 0.f;
    for (int q = 0; q < wpt; ++q) sum += red[(static_cast<size_t>(r * wpt + q) * 16 + rr) * M + m];
    // undo this CTA's power-of-two activation scale before ranks are summed:
    // each rank chose it from the max of its own K slice
    if (FMT != SB_FMT_BF16) sum = ldexpf(sum, -xshift[m]);
    tot[i] = sum;
  }
  if (ck > 1) {
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    if (rank == 0) {
      for (int i = tid; i < nrow * M; i += blockDim.x) {
        float s = tot[i];
        for (int r = 1; r < ck; ++r) s += cl.map_shared_rank(tot, r)[i];
        tot[i] = s;
      }
    }
    cl.sync();
    if (rank != 0) return;
  } else {
    __syncthreads();
  }

  // ---- 6. epilogue ----------------------------------------------------------------
  const int row0 = tile0 * 16;
  auto fin = [&](int lrow, int m) -> float {
    float v = tot[lrow * M + m];
    if (FMT == SB_FMT_NVFP4) v *= p.gscale;
    if (FMT == SB_FMT_FP8 || FMT == SB_FMT_INT8) v *= reinterpret_cast<const float*>(p.scale)[row0 + lrow];
    return v;
  };

  if (p.epi == EPI_STORE) {
    for (int i = tid; i < nrow * M; i += blockDim.x) {
      const int m = i / nrow, lrow = i % nrow, row = row0 + lrow;
      if (row < p.n) yout[static_cast<size_t>(m) * p.n + row] = f_to_bf16_bits(fin(lrow, m));
    }
  } else if (p.epi == EPI_RESID) {
    // hidden = hidden + bf16(res_mult * bf16(y))   (llm_kernels.py:306-313)
    for (int i = tid; i < nrow * M; i += blockDim.x) {
      const int m = i / nrow, lrow = i % nrow, row = row0 + lrow;
      if (row < p.n) {
        uint16_t* hp = p.y + static_cast<size_t>(m) * p.n + row;
        const float yv = bf(fin(lrow, m));
        *hp = f_to_bf16_bits(u16_to_f(*hp) + bf(p.res_mult * yv));
      }
    }
  } else if (p.epi == EPI_SWIGLU) {
    // act = bf16(bf16(silu(gate)) * up)   (llm_kernels.py:252-260); rows interleave gate/up
    const int inter = p.n / 2;
    for (int i = tid; i < (nrow / 2) * M; i += blockDim.x) {
      const int m = i / (nrow / 2), lp = i % (nrow / 2), lrow = 2 * lp, row = row0 + lrow;
      if (row < p.n) {
        const float gv = bf(fin(lrow, m));
        const float uv = bf(fin(lrow + 1, m));
        const float sg = bf(gv / (1.f + expf(-gv)));
        p.y[static_cast<size_t>(m) * inter + row / 2] = f_to_bf16_bits(sg * uv);
      }
    }
  } else if (p.epi == EPI_QKV) {
    // q/k: RoPE with each product rounded to bf16 (llm_mega.py:539-543), then
    // k/v go to cache slot ctrl[SLOT] + token (StaticLayer.update).
    const int qk_rows = (p.n_q + p.n_kv) * 128;
    const int slot_base = p.ctrl[SB_CTRL_SLOT];
    for (int i = tid; i < nrow * M; i += blockDim.x) {
      const int m = i / nrow, lrow = i % nrow, row = row0 + lrow;
      if (row >= p.n) continue;
      const int b = m / p.m_per, mi = m % p.m_per;
      const int slot = slot_base + mi;
      const bool slot_ok = slot >= 0 && slot < p.max_len;  // a replay past the cache end writes nothing
      const int head = row >> 7, within = row & 127;
      if (row < qk_rows) {
        if (within & 1) continue;  // the even row of each (j, j+64) pair does both
        const int j = within >> 1;
        int pos = slot - (p.rope_off ? p.rope_off[b] : 0);
        pos = pos < 0 ? 0 : (pos >= p.rope_max ? p.rope_max - 1 : pos);
        const float x1 = bf(fin(lrow, m));
        const float x2 = bf(fin(lrow + 1, m));
        const float cs = u16_to_f(p.cos_tab[pos * 64 + j]);
        const float sn = u16_to_f(p.sin_tab[pos * 64 + j]);
        const uint16_t o1 = f_to_bf16_bits(bf(x1 * cs) - bf(x2 * sn));
        const uint16_t o2 = f_to_bf16_bits(bf(x2 * cs) + bf(x1 * sn));
        if (head < p.n_q) {
          uint16_t* qo = p.q_out + static_cast<size_t>(m) * p.n_q * 128 + head * 128;
          qo[j] = o1;
          qo[j + 64] = o2;
        } else if (slot_ok) {
          const int kvh = head - p.n_q;
          uint16_t* kc = p.k_cache + ((static_cast<size_t>(b) * p.n_kv + kvh) * p.max_len + slot) * 128;
          kc[j] = o1;
          kc[j + 64] = o2;
        }
      } else if (slot_ok) {
        const int kvh = head - p.n_q - p.n_kv;
        p.v_cache[((static_cast<size_t>(b) * p.n_kv + kvh) * p.max_len + slot) * 128 + within] =
            f_to_bf16_bits(fin(lrow, m));
      }
    }
  } else if (p.epi == EPI_ARGMAX) {
    // logits = bf16(bf16(y) * (1/logits_scaling)), then torch argmax (first max).
    for (int m = warp; m < M; m += W) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
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
        p.part_val[static_cast<size_t>(cluster_id) * M + m] = bv;
        p.part_idx[static_cast<size_t>(cluster_id) * M + m] = bi;
      }
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
    // last CTA: reduce all partials (deterministic: total order on (value, index))
    for (int m = warp; m < M; m += W) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int q = lane; q < p.n_ctas; q += 32) {
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
      // speculative.py:430-459: accept the longest prefix where argmax == draft
      if (tid < M && p.out_ids) p.out_ids[tid] = s_best[tid];
      if (tid == 0) {
        int j = 0;
        while (j < M - 1 && static_cast<int64_t>(s_best[j]) == p.ids_io[j + 1]) ++j;
        p.ctrl[SB_CTRL_ACCEPT] = j;
      }
    } else {
      // feedback (multistep.py:181-184; batched.py:425-432: finished streams feed pad)
      for (int b = tid; b < M; b += blockDim.x) {
        const int64_t tok = s_best[b];
        int64_t out = tok, next = tok;
        if (p.finished) {
          const int f = p.finished[b];
          if (f) {
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
      if (tid == 0 && p.mode == SB_MODE_DECODE) p.ctrl[SB_CTRL_SLOT] += 1;  // position / valid_len advance
    }
    if (tid == 0) *p.counter = 0;
  }
}

// ---- host side ------------------------------------------------------------------
static const int kSMs = 148;

GemvCfg gemv_pick(int fmt, int n_pad, int k, int m) {
  GemvCfg c;
  c.nt = m <= 8 ? 1 : (m <= 16 ? 2 : (m <= 32 ? 4 : (m <= 48 ? 6 : 8)));
  const int n_tiles = n_pad / 16;
  const int kge = kgroup_elems(fmt);
  int ck = 1;
  while (ck < 8 && static_cast<long>(m) * (k / ck + 8) * 2 > 96 * 1024 && (k / (2 * ck)) % kge == 0) ck *= 2;
  while (ck < 4 && n_tiles * ck < 2 * kSMs && (k / (2 * ck)) % kge == 0 && k / (2 * ck) >= 256) ck *= 2;
  c.warps = (k / ck / kge) >= 64 ? 16 : 8;
  const int kg_cta = k / ck / kge;
  // more row tiles per CTA while: the grid stays >= 2 waves, every warp's
  // weight range still fits the register preload (<= 8 kgroups), and the
  // reduction buffers stay small
  int rt = 1;
  while (rt < 8 && rt * 2 <= c.warps && (n_tiles / (rt * 2)) * ck >= 2 * kSMs &&
         (rt * 2) * kg_cta <= 8 * c.warps && static_cast<long>(c.warps + rt * 2) * 16 * m * 4 <= 64 * 1024)
    rt *= 2;
  c.ck = ck;
  c.rt = rt;
  return c;
}

size_t gemv_smem_bytes(const GemvCfg& c, int k, int m) {
  const int k_cta = k / c.ck;
  size_t off = (static_cast<size_t>(m) * (k_cta + 8) * 2 + 15) & ~size_t(15);
  const size_t rt16 = static_cast<size_t>(c.rt) * 16;
  return off + (static_cast<size_t>(c.warps) * 16 + rt16) * m * 4 + (64 * 3 + 4 + 32) * 4 + 16;
}

int gemv_grid(const GemvCfg& c, int n_tiles) { return ((n_tiles + c.rt - 1) / c.rt) * c.ck; }

template <int FMT, int NT>
static int launch_t(const GemvParams& p, const GemvCfg& c, bool pdl, cudaStream_t stream) {
  const size_t smem = gemv_smem_bytes(c, p.k, p.m < 64 ? p.m : 64);
  int dev = 0;
  cudaGetDevice(&dev);
  static unsigned configured = 0;  // one max-dynamic-smem attribute call per (instantiation, device)
  if (!(configured & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    configured |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gemv_grid(c, p.n_tiles), (p.m + 63) / 64);
  cfg.blockDim = dim3(c.warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (c.ck > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = c.ck;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  note_launch();
  return cudaLaunchKernelEx(&cfg, k_gemv<FMT, NT>, p);
}

template <int FMT>
static int launch_fmt(const GemvParams& p, const GemvCfg& c, bool pdl, cudaStream_t s) {
  switch (c.nt) {
    case 1: return launch_t<FMT, 1>(p, c, pdl, s);
    case 2: return launch_t<FMT, 2>(p, c, pdl, s);
    case 4: return launch_t<FMT, 4>(p, c, pdl, s);
    case 6: return launch_t<FMT, 6>(p, c, pdl, s);
    case 8: return launch_t<FMT, 8>(p, c, pdl, s);
  }
  return SB_ERR_CONFIG;
}

int gemv_launch(const GemvParams& p, const GemvCfg& c, int fmt, bool pdl, cudaStream_t stream) {
  if (p.m < 1 || (p.m > 64 && (p.epi != EPI_STORE || p.pro != PRO_NONE))) return SB_ERR_CONFIG;
  if (gemv_smem_bytes(c, p.k, p.m < 64 ? p.m : 64) > 200 * 1024) return SB_ERR_CONFIG;
  switch (fmt) {
    case SB_FMT_BF16: return launch_fmt<SB_FMT_BF16>(p, c, pdl, stream);
    case SB_FMT_FP8: return launch_fmt<SB_FMT_FP8>(p, c, pdl, stream);
    case SB_FMT_INT8: return launch_fmt<SB_FMT_INT8>(p, c, pdl, stream);
    case SB_FMT_NVFP4: return launch_fmt<SB_FMT_NVFP4>(p, c, pdl, stream);
  }
  return SB_ERR_ARG;
}

}  // namespace sb
