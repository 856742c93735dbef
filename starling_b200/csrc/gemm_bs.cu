// NVFP4 block-scaled tensor-core GEMV/GEMM for 1..8 token rows, sm_100a.
//
// y[m][row] = sum_k x[m][k] * W[row][k] for NVFP4 weights (e2m1 codes, an e4m3
// scale per 16 K-elements, an fp32 tensor scale), with the prologues (RMSNorm,
// embedding) and epilogues (RoPE + KV-cache write, residual, SwiGLU, argmax)
// of the dequant-GEMV.  The mma.sync GEMV turns every code into a bf16
// fragment with ALU instructions; here the codes and their block scales go to
// the tensor core as they are (tcgen05.mma kind::mxf4nvf4.block_scale.block16,
// M = 128 weight rows per tile, K = 64 per instruction).
//
// Weight (SbLinear.w_bs): per (128-row tile, 256-element K block) one
// contiguous 18 KiB block: 16 KiB of codes (two per byte, the lower K index
// in the low nibble) in the no-swizzle K-major canonical layout of tcgen05
// (8-row x 16-byte core matrices, K chunks 128 B apart, 8-row groups 1024 B
// apart), then 2 KiB of block scales as four 512-byte chunks, one per MMA
// (64 K-elements), byte (r % 32) * 16 + (r / 32) * 4 + j for row r and
// 16-element block j: the layout tcgen05.cp .32x128b.warpx4 copies into four
// TMEM columns (row r's four scales in column r / 32 of lane r % 32, in every
// lane quarter), where the MMA reads them.
//
// Activations.  The MMA's B operand must be e2m1 with e4m3 block scales too.
// Each token row x (bf16, after the prologue) is written as a sum of
// kBsTerms = 8 e2m1 terms, each its own row of B (N = 8 per token), all with
// one power-of-two scale per 16-element block:
//   2^e >= max|x_block| / 6 (smallest such e),  y_0 = x 2^-e,
//   c_t = e2m1(y_t) (round to nearest),  y_{t+1} = 4 (y_t - c_t),
// so x = 2^e sum_t c_t 4^-t + 2^e 4^-8 y_8.  |y_0| <= 6, |y_1| <= 4,
// |y_2| <= 2, |y_t| <= 1 after, every step exact: the 8 terms reproduce each
// element to 2^-16 of 2^e (below 2^-17 of the block maximum), every bf16
// value within 2^-9 of the block maximum exactly and the rest to far below
// their bf16 ulp.  Term t's block scale is the e4m3 power of two 2^(e - E) and
// the epilogue forms sum_t D_t 2^(E - 2t), with E per token chosen so that
// 2^(e - E) <= 2^8 for every block of the CTA's K range (blocks below 2^(E-9)
// are clamped there, losing bits only 2^-17 below the largest block).
// Products of e2m1 x e4m3 values are exact, so the result differs from the
// dequantised fp32 reference only by that representation and fp32
// accumulation order.
//
// The terms are computed by the epilogue warps of every CTA for its own K
// range (the activation is at most 8 rows), straight into the resident B
// operand in shared memory: no preparation launch.
//
// Kernel (320 threads):
//  * warp 8 (one thread) streams the weight blocks into a ring of stages
//    (cp.async.bulk onto mbarriers); the first ring is issued before
//    griddepcontrol.wait, so it overlaps the previous kernel;
//  * warps 0-7 wait for the previous kernel, compute the prologue (RMSNorm
//    statistics over the whole row) and the activation terms, then run the
//    epilogue of each tile;
//  * warp 9 (one thread), once the terms are in place, copies the B scales of
//    every K block into TMEM once (tcgen05.cp), then per stage that stage's A
//    scales into the stage's own TMEM columns (so no copy rewrites columns an
//    issued MMA may still read) and issues four block-scaled MMAs into one of
//    two TMEM accumulators.
// Few tiles: a cluster of `split` (<= 8) CTAs shares a tile, each taking a
// contiguous K range, and the partial rows meet in the rank that finishes them
// (distributed shared memory, summed in rank order).  Many tiles (gate/up,
// lm_head): persistent CTAs, the epilogue of one tile overlapping the MMAs of
// the next.  Every wait is bounded; on expiry SB_CTRL_ERR = 2 is recorded.
//
// Measured on B200 (graphed launches, weights from HBM): each tcgen05.mma of
// N = 8 costs about as much as a wide one (~100 ns of issue per instruction,
// ~40 ns per tcgen05.cp) while the tensor pipe stays ~1 % busy, so a CTA
// streams ~30 GB/s; plans therefore put two CTAs (two issuing threads) on an
// SM where shared memory and TMEM allow.  With the fixed cost of a launch
// (TMEM allocation, the activation terms, ~3 us) the kernel beats the mma.sync
// GEMV on the lm_head (hundreds of tiles) and on 8-row forwards, and the host
// picks it for those shapes (api.cu).
#include <cooperative_groups.h>

#include "gemm_bs.cuh"
#include "gemv_epi.cuh"
#include "tc_common.cuh"
#include "tc_epi.cuh"

namespace cg = cooperative_groups;

namespace sb {

namespace {

__device__ __forceinline__ void tc_cp_32x128(uint32_t taddr, uint64_t sdesc_src) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc_src) : "memory");
}
__device__ __forceinline__ void bs_mma(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t tsfa,
                                       uint32_t tsfb, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(
          tmem),
      "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(tsfa), "r"(tsfb)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// smallest e with 6 * 2^e >= b (b > 0; 0 for b == 0)
__device__ __forceinline__ int bs_exp6(float b) {
  if (!(b > 0.f)) return 0;
  int ex;
  const float f = frexpf(b, &ex);  // b = f 2^ex, f in [0.5, 1)
  return f <= 0.75f ? ex - 3 : ex - 2;
}

}  // namespace

struct BsArgs {
  const uint8_t* w;  // SbLinear.w_bs
  uint32_t idesc;
  int ncol, tiles, kb, split, stages, kbc, tmem_cols, sf_col;
};

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 2) k_bs_gemm(const __grid_constant__ GemvParams p, const __grid_constant__ BsArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int M = p.m, N = a.ncol, K = p.k;
  const BsLayout L = bs_layout(N, a.kbc, a.stages, M, a.split);
  uint8_t* ring = smem;
  uint8_t* bops = smem + L.bops;
  uint8_t* sfb = smem + L.sfb;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + a.stages;
  uint64_t* acc_full = empty + a.stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* bready = acc_empty + 2;       // activation terms written
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L.tmem);
  int* s_flag = reinterpret_cast<int*>(smem + L.flag);
  int* s_gexp = reinterpret_cast<int*>(smem + L.gexp);
  float* s_rstd = reinterpret_cast<float*>(smem + L.rstd);
  int* s_amax = reinterpret_cast<int*>(smem + L.amax);
  float* s_red = reinterpret_cast<float*>(smem + L.red);
  int* s_best = reinterpret_cast<int*>(smem + L.best);
  float* s_bval = reinterpret_cast<float*>(smem + L.bval);
  float* wb_val = reinterpret_cast<float*>(smem + L.wbv);
  int* wb_idx = reinterpret_cast<int*>(smem + L.wbi);
  float* part = reinterpret_cast<float*>(smem + L.part);
  int32_t* err = p.ctrl ? p.ctrl + SB_CTRL_ERR : nullptr;

  const int S = a.split;
  const int q = S > 1 ? static_cast<int>(cg::this_cluster().block_rank()) : 0;
  const int cid = blockIdx.x / S, ncl = gridDim.x / S;
  const int kb0 = q * a.kb / S, kb1 = (q + 1) * a.kb / S, nk = kb1 - kb0;  // nk >= 1: split <= kb
  const int my_tiles = cid < a.tiles ? (a.tiles - cid + ncl - 1) / ncl : 0;
  const int rot = cid % nk;  // CTAs start their K loop at different blocks

  constexpr int kProd = kTcEpiWarps, kMma = kTcEpiWarps + 1;
  if (warp == kProd && lane == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(acc_full + b2, 1);
      mbar_init(acc_empty + b2, kTcEpiWarps * 32);
    }
    mbar_init(bready, 1);
    mbar_fence_init();
  }
  if (warp == kMma) tmem_alloc(s_tmem, static_cast<uint32_t>(a.tmem_cols));
  if constexpr (EPI == EPI_ARGMAX)
    for (int i = tid; i < (kTcEpiWarps + 2) * 128; i += blockDim.x) {
      wb_val[i] = -INFINITY;
      wb_idx[i] = 0x7fffffff;
    }
  if (tid < kBsMaxRows) s_amax[tid] = 0;
  // B scale chunks: rows the MMA does not read are zero, not leftovers (written
  // by the warps that later fence their writes for the tensor core)
  if (warp < kTcEpiWarps)
    for (int i = tid; i < nk * 2048 / 16; i += kTcEpiWarps * 32) reinterpret_cast<uint4*>(sfb)[i] = make_uint4(0, 0, 0, 0);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == kProd) {
    // ---- producer: weight blocks only (the activation terms are built here) ----
    if (lane == 0) {
      const int total = my_tiles * nk;
      auto a_src = [&](int it) {
        const int t = cid + (it / nk) * ncl;
        const int kb = kb0 + (it % nk + rot) % nk;
        return a.w + (static_cast<size_t>(t) * a.kb + kb) * kBsBlock;
      };
      const int pre = total < a.stages ? total : a.stages;
      for (int it = 0; it < pre; ++it) {  // weights do not depend on the previous kernel
        mbar_expect_tx(full + it, kBsBlock);
        bulk_g2s(ring + static_cast<size_t>(it) * kBsBlock, a_src(it), kBsBlock, full + it);
      }
      for (int it = pre; it < total; ++it) {
        const int s = it % a.stages;
        wait_bounded(empty + s, static_cast<uint32_t>((it / a.stages - 1) & 1), err);
        mbar_expect_tx(full + s, kBsBlock);
        bulk_g2s(ring + static_cast<size_t>(s) * kBsBlock, a_src(it), kBsBlock, full + s);
      }
    }
    __syncwarp();
    pdl_wait();
    pdl_launch();
  } else if (warp == kMma) {
    // ---- MMA issuer ----
    pdl_wait();
    pdl_launch();
    if (lane == 0) {
      wait_bounded(bready, 0, err);
      tc_fence_after();
      // TMEM scale columns: A per ring stage (16 each), B per K block of this
      // CTA (16 each, copied once: the terms are the same for every tile)
      const uint32_t tsfa = tmem + static_cast<uint32_t>(a.sf_col);
      const uint32_t tsfb = tsfa + static_cast<uint32_t>(16 * a.stages);
      const uint32_t sb0 = su32(bops), sf0 = su32(sfb);
      for (int kbl = 0; kbl < nk; ++kbl)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 32 rows x 16 bytes, 8-row core matrices 128 B apart
          tc_cp_32x128(tsfb + static_cast<uint32_t>(16 * kbl + 4 * kk),
                       sdesc(sf0 + static_cast<uint32_t>(kbl * 2048 + kk * 512), 0u, 128u));
      int it = 0;
      for (int tc = 0; tc < my_tiles; ++tc) {
        const int buf = tc & 1;
        if (tc >= 2) wait_bounded(acc_empty + buf, static_cast<uint32_t>((tc / 2 - 1) & 1), err);
        tc_fence_after();
        const uint32_t dacc = tmem + static_cast<uint32_t>(buf * N);
        for (int j = 0; j < nk; ++j, ++it) {
          const int s = it % a.stages;
          const int kbl = (j + rot) % nk;  // the K block the producer put in this stage
          wait_bounded(full + s, static_cast<uint32_t>((it / a.stages) & 1), err);
          tc_fence_after();
          const uint32_t sa = su32(ring + static_cast<size_t>(s) * kBsBlock);
          const uint32_t sbb = sb0 + static_cast<uint32_t>(kbl * N * 128);
          const uint32_t ta = tsfa + static_cast<uint32_t>(16 * s), tb = tsfb + static_cast<uint32_t>(16 * kbl);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) tc_cp_32x128(ta + 4u * kk, sdesc(sa + kBsCodeBytes + kk * 512u, 0u, 128u));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            bs_mma(dacc, sdesc(sa + kk * 256u, 128u, 1024u), sdesc(sbb + kk * 256u, 128u, 1024u), a.idesc,
                   ta + 4u * kk, tb + 4u * kk, (j > 0 || kk > 0) ? 1u : 0u);
          tc_commit(empty + s);  // the stage is free once these MMAs have read it
        }
        tc_commit(acc_full + buf);
      }
    }
    __syncwarp();
  } else {
    // ---- warps 0-7: activation terms, then the epilogue ----
    pdl_wait();
    pdl_launch();
    const bool embed = p.pro == PRO_EMBED;
    auto row_src = [&](int m) -> const uint16_t* {
      if (embed) {
        int64_t id = p.ids[m];
        id = id < 0 ? 0 : (id >= p.embed_rows ? p.embed_rows - 1 : id);  // never read outside the table
        return p.embed + static_cast<size_t>(id) * K;
      }
      return p.x + static_cast<size_t>(m) * K;
    };
    const int k0 = kb0 * 256, Kc = nk * 256;
    // 8 prologue values of token m at element k into f (RMSNorm applied once
    // s_rstd is ready)
    auto load_vals = [&](int m, int k, float* f) {
      unpack8(*reinterpret_cast<const uint4*>(row_src(m) + k), f);
      if (embed)
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = bf(f[e] * p.emb_mult);
      if (p.pro != PRO_NONE) {  // weight * bf16(x * rstd)
        float wn[8];
        unpack8(__ldg(reinterpret_cast<const uint4*>(p.norm_w + k)), wn);
        const float rs = s_rstd[m];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = bf(wn[e] * bf(f[e] * rs));
      }
    };
    // Pass A: the token exponent E (term scales 2^(E - 2t)).  With RMSNorm
    // (modeling_granite.py:192-197) the statistics read the whole row, and the
    // same pass bounds the normalised values of this CTA's range:
    // |w bf16(x rstd)| <= |w x| rstd (1 + 2^-6).  The embedded rows
    // (embed_tokens(ids) * 12, llm_mega.py:514) are written out once, by CTA 0.
    if (p.pro != PRO_NONE) {
      float ss[kBsMaxRows], mw[kBsMaxRows];
#pragma unroll
      for (int m = 0; m < kBsMaxRows; ++m) {
        ss[m] = 0.f;
        mw[m] = 0.f;
        if (m < M) {
          const uint16_t* src = row_src(m);
          for (int c = tid; c < K / 8; c += kTcEpiWarps * 32) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4*>(src + c * 8), f);
            if (embed) {
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = bf(f[e] * p.emb_mult);
              if (p.hidden_out && blockIdx.x == 0)
                *reinterpret_cast<uint4*>(p.hidden_out + static_cast<size_t>(m) * K + c * 8) = pack8(f);
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) ss[m] += f[e] * f[e];
            if (c * 8 >= k0 && c * 8 < k0 + Kc) {
              float wn[8];
              unpack8(__ldg(reinterpret_cast<const uint4*>(p.norm_w + c * 8)), wn);
#pragma unroll
              for (int e = 0; e < 8; ++e) mw[m] = fmaxf(mw[m], fabsf(wn[e] * f[e]));
            }
          }
        }
      }
#pragma unroll
      for (int m = 0; m < kBsMaxRows; ++m) {
        const float v = warp_sum(ss[m]), w = warp_max(mw[m]);
        if (lane == 0) {
          s_red[warp * kBsMaxRows + m] = v;
          s_red[64 + warp * kBsMaxRows + m] = w;
        }
      }
      epi_sync();
      if (tid < M) {
        float t = 0.f, w = 0.f;
        for (int i = 0; i < kTcEpiWarps; ++i) {
          t += s_red[i * kBsMaxRows + tid];
          w = fmaxf(w, s_red[64 + i * kBsMaxRows + tid]);
        }
        const float rs = 1.f / sqrtf(t / static_cast<float>(K) + p.eps);
        s_rstd[tid] = rs;
        s_gexp[tid] = bs_exp6(w * rs * (1.f + 0.015625f)) - 8;
      }
      epi_sync();
    } else {
      // items: (token, 8 consecutive elements of the CTA's K range); per token
      // 32 * nk items, so a warp's 32 items always belong to one token
      for (int it = tid; it < M * nk * 32; it += kTcEpiWarps * 32) {
        const int m = it / (nk * 32), e0 = (it % (nk * 32)) * 8;
        float f[8];
        load_vals(m, k0 + e0, f);
        float mx = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(f[e]));
        mx = warp_max(mx);
        if (lane == 0) atomicMax(s_amax + m, __float_as_int(mx));  // non-negative: int order = float order
      }
      epi_sync();
      if (tid < M) s_gexp[tid] = bs_exp6(__int_as_float(s_amax[tid])) - 8;
      epi_sync();
    }
    // Pass B: the terms.  Per 16-element block (two adjacent lanes, 8 elements
    // each) one power-of-two scale 2^e >= max / 6, clamped to 2^(E-9)..2^(E+8)
    // (its e4m3 byte 2^(e-E) is every term's block scale); y = x 2^-e, then
    // per term c = e2m1(y), y = 4 (y - c): all exact.
    for (int it = tid; it < M * nk * 32; it += kTcEpiWarps * 32) {
      const int m = it / (nk * 32), e0 = (it % (nk * 32)) * 8;
      float y[8];
      load_vals(m, k0 + e0, y);
      float bm = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) bm = fmaxf(bm, fabsf(y[e]));
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));  // the block's other half
      const int E = s_gexp[m];
      int eb2 = bm > 0.f ? bs_exp6(bm) : E - 9;
      eb2 = eb2 < E - 9 ? E - 9 : (eb2 > E + 8 ? E + 8 : eb2);
      const int d = eb2 - E;  // -9..8: e4m3 2^d, subnormal below 2^-6
      const uint8_t s8 = static_cast<uint8_t>(d >= -6 ? (d + 7) << 3 : 1 << (d + 9));
      // x 2^-eb2: an exact multiply when 2^-eb2 is a normal float (the same
      // result as ldexpf, which stays for the extreme exponents)
      const bool fast = eb2 >= -126 && eb2 <= 126;
      const float sc = fast ? __int_as_float((127 - eb2) << 23) : 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = fast ? y[e] * sc : ldexpf(y[e], -eb2);
      const int kbl = e0 >> 8, eb = e0 & 255;         // K block of the CTA range, element within it
      const int kbyte = eb >> 1;                       // byte of the 128-byte row (4-byte aligned)
      const int kstep = eb >> 6, blk = (eb >> 4) & 3;  // MMA of the block (64 elements), 16-element block
      const bool first_half = (eb & 8) == 0;
      uint8_t* bo = bops + static_cast<size_t>(kbl) * N * 128 + (kbyte >> 4) * 128 + (kbyte & 15);
      uint8_t* so = sfb + kbl * 2048 + kstep * 512 + blk;
#pragma unroll
      for (int t = 0; t < kBsTerms; ++t) {
        uint32_t codes = 0;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const __nv_fp4x2_storage_t c2 =
              __nv_cvt_float2_to_fp4x2(make_float2(y[2 * jj], y[2 * jj + 1]), __NV_E2M1, cudaRoundNearest);
          codes |= static_cast<uint32_t>(c2) << (8 * jj);
          const __half2_raw h = __nv_cvt_fp4x2_to_halfraw2(c2, __NV_E2M1);
          y[2 * jj] = (y[2 * jj] - __half2float(__half(__half_raw{h.x}))) * 4.f;
          y[2 * jj + 1] = (y[2 * jj + 1] - __half2float(__half(__half_raw{h.y}))) * 4.f;
        }
        const int n = m * kBsTerms + t;  // B row
        *reinterpret_cast<uint32_t*>(bo + (n >> 3) * 1024 + (n & 7) * 16) = codes;
        if (first_half) so[(n & 31) * 16 + (n >> 5) * 4] = s8;
      }
    }
    fence_proxy_async();  // the generic-proxy writes above are read by tcgen05.cp / tcgen05.mma
    epi_sync();
    if (tid == 0) mbar_arrive(bready);
    // bring the epilogue's global inputs into L1 while the MMAs run: the
    // residual rows this CTA finishes, the RoPE rows at each token's position
    if constexpr (EPI == EPI_RESID) {
      const int rp0 = tc_rows_per_rank(S);
      const int ra = cid * 128 + (S > 1 ? q * rp0 : 0), nr = S > 1 ? rp0 : 128;
      const int rb = min(ra + nr, p.n);
      const int nseg = (rb - ra + 63) / 64;  // 128-byte lines of bf16 rows
      for (int i = tid; i < M * nseg; i += kTcEpiWarps * 32)
        if (ra < rb)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(p.y + static_cast<size_t>(i / nseg) * p.n + ra + (i % nseg) * 64));
    } else if constexpr (EPI == EPI_QKV) {
      const int slot_base = p.ctrl[SB_CTRL_SLOT];
      for (int i = tid; i < M; i += kTcEpiWarps * 32) {
        const int b = i / p.m_per;
        int pos = slot_base + i % p.m_per - (p.rope_off ? p.rope_off[b] : 0);
        pos = pos < 0 ? 0 : (pos >= p.rope_max ? p.rope_max - 1 : pos);
        asm volatile("prefetch.global.L1 [%0];" ::"l"(p.cos_tab + static_cast<size_t>(pos) * 64));
        asm volatile("prefetch.global.L1 [%0];" ::"l"(p.sin_tab + static_cast<size_t>(pos) * 64));
      }
    }

    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4).. (tile rows); warps 0-3
    // take tokens 0-3, warps 4-7 tokens 4-7 ----
    const int lq = warp & 3, m0 = (warp >> 2) * 4;
    const int lrow = lq * 32 + lane;
    const int rp = tc_rows_per_rank(S), ms = tc_inbox_stride(M);
    for (int tc = 0; tc < my_tiles; ++tc) {
      const int t = cid + tc * ncl, buf = tc & 1;
      const uint32_t taddr = tmem + static_cast<uint32_t>(buf * N) + (static_cast<uint32_t>(lq * 32) << 16);
      wait_bounded(acc_full + buf, static_cast<uint32_t>((tc / 2) & 1), err);
      tc_fence_after();
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (m0 < M) {
        uint32_t d[4][8];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (m0 + i < M) tmem_ld8(taddr + static_cast<uint32_t>((m0 + i) * kBsTerms), d[i]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (m0 + i < M) {
            const int E = s_gexp[m0 + i];
            float acc = 0.f;
#pragma unroll
            for (int tt = 0; tt < kBsTerms; ++tt) {
              const int e2 = E - 2 * tt;  // 2^e2 exactly: bit pattern when normal, else ldexpf
              const float w2 = e2 >= -126 && e2 <= 127 ? __int_as_float((e2 + 127) << 23) : ldexpf(1.f, e2);
              acc = fmaf(__uint_as_float(d[i][tt]), w2, acc);
            }
            v[i] = acc;
          }
      }
      tc_fence_before();
      mbar_arrive(acc_empty + buf);  // the MMA warp may overwrite this accumulator
      if (m0 < M) {
        if (S == 1) {
          const int row = t * 128 + lrow;
          tc_epi<SB_FMT_NVFP4, 4, EPI>(p, row, row < p.n, v, m0, M, wb_val, wb_idx, warp, 0);
        } else {
          // push this K partial to the rank that finishes the row (16-byte DSMEM store)
          float* dst = cg::this_cluster().map_shared_rank(part, lrow / rp) + (q * rp + lrow % rp) * ms + m0;
          *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    }
  }

  if (S > 1) {  // one tile per cluster: sum the pushed K partials in rank order, then the epilogue
    cg::this_cluster().sync();
    const int rp = tc_rows_per_rank(S), r0 = q * rp, ms = tc_inbox_stride(M);
    const int nr = r0 >= 128 ? 0 : (r0 + rp > 128 ? 128 - r0 : rp);
    const int nw = blockDim.x >> 5, ngrp = (nr + 31) / 32, nch = (M + 3) / 4;
    for (int item = warp; item < ngrp * nch; item += nw) {
      const int rg = item / nch, c0 = (item % nch) * 4;
      const int lr = rg * 32 + lane;
      const bool ok = lr < nr;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok)
        for (int c = 0; c < S; ++c) {
          const float4 x4 = *reinterpret_cast<const float4*>(part + (c * rp + lr) * ms + c0);
          v[0] += x4.x;
          v[1] += x4.y;
          v[2] += x4.z;
          v[3] += x4.w;
        }
      const int row = cid * 128 + r0 + lr;
      tc_epi<SB_FMT_NVFP4, 4, EPI>(p, row, ok && row < p.n, v, c0, M, wb_val, wb_idx, warp, 0);
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {  // combine the warps' running bests (order-independent total order)
    __syncthreads();
    for (int m = tid; m < M; m += blockDim.x) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int w = 0; w < kTcEpiWarps + 2; ++w)
        if (am_better(wb_val[w * 128 + m], wb_idx[w * 128 + m], bv, bi)) {
          bv = wb_val[w * 128 + m];
          bi = wb_idx[w * 128 + m];
        }
      s_bval[m] = bv;
      s_best[m] = bi;
    }
  }
  __syncthreads();
  if constexpr (EPI == EPI_ARGMAX) gemv_argmax_finish(p, s_best, s_bval, M, my_tiles > 0, s_flag);
  tc_fence_before();
  __syncthreads();
  if (warp == kMma) {
    tc_fence_after();
    tmem_dealloc(tmem, static_cast<uint32_t>(a.tmem_cols));
  }
}

// ---- host side ------------------------------------------------------------------
static const int kSMs = 148;
static const size_t kBsSmemOne = 220 * 1024;  // one CTA per SM (persistent over tiles)
static const size_t kBsSmemTwo = 110 * 1024;  // two CTAs per SM (clusters splitting K)

static int bs_ctas_per_sm_max() { return 2; }

// Plan for per_sm CTAs per SM (1: up to 220 KB of shared memory and 512 TMEM
// columns each; 2: half of both).  Two CTAs per SM run two MMA-issuing threads
// per SM, which is what bounds this kernel (tcgen05 issue latency, not the
// tensor pipe): lm_head at 1 row 34.4 -> 24.7 us, gate/up at 8 rows 26.1 ->
// 18.9 us on B200.
static bool bs_plan_for(int n, int k, int m, int per_sm, BsPlan& pl) {
  pl.m = m;
  pl.ncol = kBsTerms * m;
  pl.tiles = (n + 127) / 128;
  pl.kb = k / 256;
  const int slots = kSMs * per_sm;
  if (pl.tiles * 4 >= slots * 3) {  // enough tiles: persistent, no K split
    pl.split = 1;
    pl.n_ctas = pl.tiles < slots ? pl.tiles : slots;
  } else {
    int s = slots / pl.tiles;
    if (s > 8) s = 8;
    if (s > pl.kb) s = pl.kb;
    if (s < 1) s = 1;
    pl.split = s;
    pl.n_ctas = pl.tiles * s;
  }
  const bool two = pl.split > 1 || per_sm > 1;  // two CTAs per SM
  pl.kbc = (pl.kb + pl.split - 1) / pl.split;
  const int acc = 2 * pl.ncol;
  pl.sf_col = (acc + 31) / 32 * 32;
  // TMEM: accumulators, then 16 scale columns per ring stage (A) and per K
  // block (B)
  const int tmem_max = two ? 256 : 512;
  const size_t budget = two ? kBsSmemTwo : kBsSmemOne;
  int max_st = pl.split > 1 ? pl.kbc : 12;  // a split CTA has at most kbc blocks: all in flight at once
  if (max_st > 12) max_st = 12;
  pl.stages = 0;
  for (int st = max_st; st >= 1; --st)
    if (bs_layout(pl.ncol, pl.kbc, st, m, pl.split).total <= budget && pl.sf_col + 16 * (st + pl.kbc) <= tmem_max) {
      pl.stages = st;
      break;
    }
  if (!pl.stages) return false;
  pl.tmem_cols = 32;
  while (pl.tmem_cols < pl.sf_col + 16 * (pl.stages + pl.kbc)) pl.tmem_cols *= 2;
  pl.smem = bs_layout(pl.ncol, pl.kbc, pl.stages, m, pl.split).total;
  return true;
}

bool bs_plan(int n, int k, int m, BsPlan& pl) {
  if (m < 1 || m > kBsMaxRows || n < 1 || k < 256 || k % 256 != 0) return false;
  if (bs_ctas_per_sm_max() >= 2 && bs_plan_for(n, k, m, 2, pl)) return true;
  return bs_plan_for(n, k, m, 1, pl);
}

template <int EPI>
static int bs_launch_t(const cudaLaunchConfig_t& cfg, const GemvParams& p, const BsArgs& a) {
  int dev = 0;
  cudaGetDevice(&dev);
  static unsigned configured = 0;
  if (!(configured & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(k_bs_gemm<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kBsSmemOne));
    if (e != cudaSuccess) return e;
    configured |= 1u << dev;
  }
  return cudaLaunchKernelEx(&cfg, k_bs_gemm<EPI>, p, a);
}

int bs_launch(const GemvParams& p0, const void* w_bs, const BsPlan& pl, bool pdl, cudaStream_t stream) {
  GemvParams p = p0;
  p.n_ctas = pl.n_ctas;
  BsArgs a;
  a.w = static_cast<const uint8_t*>(w_bs);
  // instruction descriptor: A, B e2m1 (format 1) K-major; N >> 3 at bit 17; ue4m3
  // scales (bit 23 = 0); M = 128 (>> 4, bit 24); scale-factor ids 0; K = 64
  a.idesc = (1u << 7) | (1u << 10) | (static_cast<uint32_t>(pl.ncol >> 3) << 17) | ((128u >> 4) << 24);
  a.ncol = pl.ncol;
  a.tiles = pl.tiles;
  a.kb = pl.kb;
  a.split = pl.split;
  a.stages = pl.stages;
  a.kbc = pl.kbc;
  a.tmem_cols = pl.tmem_cols;
  a.sf_col = pl.sf_col;

  cudaLaunchAttribute at[2];
  int na = 0;
  if (pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (pl.split > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = pl.split;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_ctas);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cfg.attrs = at;
  cfg.numAttrs = na;
  note_launch();
  switch (p.epi) {
    case EPI_STORE: return bs_launch_t<EPI_STORE>(cfg, p, a);
    case EPI_QKV: return bs_launch_t<EPI_QKV>(cfg, p, a);
    case EPI_RESID: return bs_launch_t<EPI_RESID>(cfg, p, a);
    case EPI_SWIGLU: return bs_launch_t<EPI_SWIGLU>(cfg, p, a);
    case EPI_ARGMAX: return bs_launch_t<EPI_ARGMAX>(cfg, p, a);
  }
  return SB_ERR_ARG;
}

}  // namespace sb
