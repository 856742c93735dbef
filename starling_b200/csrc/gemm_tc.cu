// Tensor-core skinny GEMM for 9..128 token rows (batched decode, speculative
// verify, prefill chunks), sm_100a: tcgen05.mma with the accumulator in TMEM.
//
// y[m][row] = sum_k x[m][k] * W[row][k] with the same fused prologues
// (RMSNorm, embedding) and epilogues (RoPE + KV-cache write, residual,
// SwiGLU, argmax + token feedback) as the dequant-GEMV.  The weight rows are
// the MMA's M side (128 rows per tile), the tokens its N side.
//
// Operands.  The weight is read from its tensor-core tile copy (SbLinear.w_tc):
// for every (128-row tile, 128-byte K block) one contiguous 16 KiB block in
// the canonical no-swizzle K-major layout of tcgen05 (8-row x 16-byte core
// matrices; K chunks 128 B apart, 8-row groups 1024 B apart), so one bulk
// copy (cp.async.bulk, no tensor map) stages it.  The activations are
// prepared once per launch (k_tc_prep_cta / k_tc_prep_warp) into the same layout:
//  * bf16 weights (kind::f16): the bf16 rows themselves (after the prologue);
//  * fp8 weights (kind::f8f6f4, e4m3 x e4m3): each row is scaled by a power
//    of two 2^s (max |x| 2^s in [128, 256)) and split into two e4m3 terms,
//    x 2^s = t0 + t1/16 with t0 = e4m3(x 2^s), t1 = e4m3(16 (x 2^s - t0)).
//    Both subtractions are exact, and the pair represents every bf16 value
//    within 2^13 of the row maximum exactly (smaller ones to 2^-14 absolute
//    in the scaled units).  The two terms are the two halves of the MMA's N
//    (columns m and mp + m); the epilogue forms (D0 + D1/16) 2^-s.  Products
//    of e4m3 values are exact, so the result differs from the dequantised
//    fp32 reference only by fp32 accumulation order.
//
// Decode chain (OPB = 1, fp8 weights, 9..64 token rows): no preparation.
// The preceding GEMM's epilogue wrote a block-scaled operand (operand.cuh):
// the same two e4m3 terms, with one UE8M0 scale per (token, 32 elements) in
// place of a whole-row shift, and the RMSNorm weight already applied.
//  * The MMA is kind::mxf8f6f4.block_scale.  Each stage's 512 bytes of B
//    scales go to the stage's own four TMEM columns (tcgen05.cp), the
//    weight's scales are a constant 1.0, and MMA kk of a stage selects byte
//    kk of the scale words through the descriptor's scale ids.
//  * The epilogue applies the token's RMSNorm 1 / rms, summed from the
//    producer's per-32-row sums of squares.
//  * Producers: the residual epilogue (o, down) stages each finishing warp's
//    32 new rows x 4 tokens in shared memory and writes whole blocks; the
//    SwiGLU epilogue (gate/up, no K split) stages its tile's 64 activations
//    of every token and writes them with all epilogue warps.
//
// Kernel (NEPI epilogue warps + 2: 16 + 2 with one CTA per SM, 8 + 2 with two):
//  * warp NEPI (one thread) streams (A block, B block) pairs into a ring of
//    shared-memory stages with bulk copies completing on mbarriers; the weight
//    blocks of the first ring are issued BEFORE griddepcontrol.wait, so they
//    overlap the previous kernel.  CTAs start their K loop at different
//    blocks so that they do not all read the same activation block from L2;
//  * warp NEPI + 1 (one thread) issues four tcgen05.mma (K = 32 bytes each)
//    per stage into one of two TMEM accumulators and frees the stage with
//    tcgen05.commit;
//  * warps 0..NEPI-1 read the 128 x N fp32 accumulator (warp w reads TMEM
//    lanes 32 (w % 4).. = tile rows; the NEPI / 4 warps of a lane quarter
//    interleave over 8-token chunks), undo the activation scaling and run the
//    fused row-owned epilogue (tc_epi.cuh).  Sixteen warps keep a 128-token
//    prefill tile's epilogue shorter than its MMAs.
// With many tiles (lm_head, gate/up) each CTA is persistent over tiles and the
// epilogue of one tile overlaps the MMAs of the next (double-buffered
// accumulator; with one token tile and hundreds of weight tiles, two CTAs of
// <= 110 KB per SM).  With few tiles a cluster of `split` (<= 4) CTAs shares a
// tile, each taking a contiguous K range; every CTA pushes its partial rows
// to the rank that finishes them (distributed shared memory), which sums them
// in rank order (deterministic) and runs the epilogue on 128/split rows.
// Every wait is bounded (2 s of %globaltimer); on expiry the kernel records
// SB_CTRL_ERR = 2 and carries on with invalid results instead of hanging.
#include <atomic>
#include <cooperative_groups.h>

#include "gemm_tc.cuh"
#include "operand.cuh"
#include "tc_common.cuh"
#include "gemv_epi.cuh"
#include "tc_epi.cuh"

namespace cg = cooperative_groups;

namespace sb {

namespace {

__device__ __forceinline__ void tc_fence_proxy_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 128 rows x 4 bytes of scales from shared memory into four TMEM columns
// (row r in column r / 32 of lane r % 32, in every lane quarter)
__device__ __forceinline__ void tc_cp_scales(uint32_t taddr, uint64_t src) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src) : "memory");
}
// e4m3 x e4m3 with a UE8M0 scale per 32 K-elements of each A and B row; the
// byte of each scale word used is chosen by the descriptor's scale ids
__device__ __forceinline__ void tc_mma_mx8(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t tsfa,
                                          uint32_t tsfb, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}\n" ::"r"(tmem),
      "l"(ad), "l"(bd), "r"(idesc), "r"(acc), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// fixed-order block reductions over 256 threads
__device__ __forceinline__ float block_sum256(float v, float* s_red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t += s_red[i];
  __syncthreads();
  return t;
}
__device__ __forceinline__ float block_max256(float v, float* s_red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) t = fmaxf(t, s_red[i]);
  __syncthreads();
  return t;
}

}  // namespace

struct TcArgs {
  const uint8_t* wt;      // weight tiles [tiles][kb][16 KiB]
  const uint8_t* xq;      // B operand [kb][np/8][8 chunks][8 rows][16 B]
  const int32_t* xshift;  // fp8: per-row power-of-two scale of the activations
  uint32_t idesc;
  int mp, np, tiles, kb, split, stages, ncols;
  int mtiles;  // token tiles of mp rows (EPI_STORE only when > 1: prefill projections)
  int rank_shift;  // fp8: xshift holds one row of shifts per K-split rank (operand written per rank)
  // block-scaled operand (OPB): TMEM columns allocated; first column of the
  // weight's scales (4) and of the B scales (4 per stage)
  int tmem_cols, sfa_col, sfb_col;
};

// ---- B operand: prologue + layout ------------------------------------------------
// Many rows (prefill, token tiles of 128): one warp per (padded) token row,
// kPrepRows rows per CTA: every reduction is a warp shuffle (no block barrier),
// every lane works at any K, and the rows keep the SMs busy.  Lane l takes
// the 16-element chunks l, l + 32, ... of the row; the row is read in up to
// three passes (RMSNorm statistics; the maximum for the fp8 scale; the
// output), the later ones from L1.  Rows >= m and padding rows of right-padded
// prompts are written as zeros.
constexpr int kPrepRows = 8;
constexpr int kPrepThreads = kPrepRows * 32;
constexpr int kPrepMaxK = 16384;

template <int FMT>
__global__ void __launch_bounds__(kPrepThreads) k_tc_prep_warp(const __grid_constant__ GemvParams p, uint8_t* xq,
                                                                int32_t* xshift, int mp, int np, int rows) {
  const int lane = threadIdx.x & 31;
  const int m = blockIdx.x * kPrepRows + (threadIdx.x >> 5);  // token (padded to whole token tiles)
  const int K = p.k, n16 = K / 16;
  const size_t kb_bytes = static_cast<size_t>(np) * 128;
  constexpr int CPE = tc_bf16_operand(FMT) ? 2 : 1;  // 16-byte output chunks per 16 elements and term
  if (p.pro != PRO_NONE && m < p.m)  // RMSNorm weights are constant: warm L1 before the dependency wait
    for (int c16 = lane; c16 < n16; c16 += 32) asm volatile("prefetch.global.L1 [%0];" ::"l"(p.norm_w + c16 * 16));
  pdl_wait();
  pdl_launch();
  if (m >= rows) return;
  // token tile m / mp holds rows mp * tile .. of the operand, each tile [kb][np/8][8][8][16 B]
  uint8_t* xt = xq + static_cast<size_t>(m / mp) * (K * (tc_bf16_operand(FMT) ? 2 : 1) / 128) * kb_bytes;
  const int ml = m % mp;  // row of the token within its tile
  auto off = [&](int n, int c) -> size_t {  // 16-byte chunk c (along K bytes) of B-operand row n
    return static_cast<size_t>(c >> 3) * kb_bytes + static_cast<size_t>(n >> 3) * 1024 + (c & 7) * 128 + (n & 7) * 16;
  };
  const bool pad_row = m < p.m && p.row_len && (m % p.row_T) >= p.row_len[p.row_b0 + m / p.row_T];
  if (m >= p.m || pad_row) {  // past the tokens, or a prompt's padding: zero operand rows
    for (int c = lane; c < n16 * CPE; c += 32) {
      *reinterpret_cast<uint4*>(xt + off(ml, c)) = make_uint4(0, 0, 0, 0);
      if (FMT == SB_FMT_FP8) *reinterpret_cast<uint4*>(xt + off(mp + ml, c)) = make_uint4(0, 0, 0, 0);
    }
    if (FMT == SB_FMT_FP8 && lane == 0) xshift[m] = 0;
    return;
  }
  const bool embed = p.pro == PRO_EMBED;
  const uint16_t* src;
  if (embed) {
    int64_t id = p.ids[m];
    id = id < 0 ? 0 : (id >= p.embed_rows ? p.embed_rows - 1 : id);  // never read outside the table
    src = p.embed + static_cast<size_t>(id) * K;
  } else {
    src = p.x + static_cast<size_t>(m) * K;
  }
  // the 16 input values of chunk c16 (embedding rows: embed_tokens(ids) * 12, llm_mega.py:514)
  auto load16 = [&](int c16, float* f) {
    unpack8(*reinterpret_cast<const uint4*>(src + c16 * 16), f);
    unpack8(*reinterpret_cast<const uint4*>(src + c16 * 16 + 8), f + 8);
    if (embed)
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = bf(f[e] * p.emb_mult);
  };
  float rstd = 0.f;
  if (p.pro != PRO_NONE) {  // RMSNorm statistics (modeling_granite.py:192-197)
    float ss = 0.f;
    for (int c16 = lane; c16 < n16; c16 += 32) {
      float f[16];
      load16(c16, f);
      if (embed && p.hidden_out) {  // the residual stream of layer 0
        uint4* ho = reinterpret_cast<uint4*>(p.hidden_out + static_cast<size_t>(m) * K + c16 * 16);
        ho[0] = pack8(f);
        ho[1] = pack8(f + 8);
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) ss += f[e] * f[e];
    }
    ss = warp_sum(ss);
    rstd = 1.f / sqrtf(ss / static_cast<float>(K) + p.eps);
  }
  // prologue output of chunk c16: weight * bf16(x * rstd), or the input
  auto values16 = [&](int c16, float* f) {
    load16(c16, f);
    if (p.pro != PRO_NONE) {
      float wn[16];
      unpack8(__ldg(reinterpret_cast<const uint4*>(p.norm_w + c16 * 16)), wn);
      unpack8(__ldg(reinterpret_cast<const uint4*>(p.norm_w + c16 * 16 + 8)), wn + 8);
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = bf(wn[e] * bf(f[e] * rstd));
    }
  };
  if constexpr (tc_bf16_operand(FMT)) {
    for (int c16 = lane; c16 < n16; c16 += 32) {
      float f[16];
      values16(c16, f);
      *reinterpret_cast<uint4*>(xt + off(ml, 2 * c16)) = pack8(f);
      *reinterpret_cast<uint4*>(xt + off(ml, 2 * c16 + 1)) = pack8(f + 8);
    }
  } else {
    float am = 0.f;
    for (int c16 = lane; c16 < n16; c16 += 32) {
      float f[16];
      values16(c16, f);
#pragma unroll
      for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(f[e]));
    }
    am = warp_max(am);
    int e2 = 0;
    if (am > 0.f) frexpf(am, &e2);
    const int shift = 8 - e2;  // max |x| 2^shift in [128, 256)
    if (lane == 0) xshift[m] = shift;
    for (int c16 = lane; c16 < n16; c16 += 32) {
      float f[16];
      values16(c16, f);
      uint4 w0, w1;
      e4m3_split16(f, shift, w0, w1);
      *reinterpret_cast<uint4*>(xt + off(ml, c16)) = w0;
      *reinterpret_cast<uint4*>(xt + off(mp + ml, c16)) = w1;
    }
  }
}

// Many rows, K a multiple of 2048 up to 16384 (prefill): each row is held in
// registers, one warp per 2048-element section (lane l: 16-element chunks
// l, l + 32, l + 64, l + 96 of the section, all loaded before any is used),
// S = K / 2048 warps per row and 8 / S rows per CTA.  Every input element is
// read once; the RMSNorm sum of squares and the fp8 maximum are warp shuffles,
// combined over a row's S warps through shared memory in section order.
constexpr int kRowsChunks = 4;  // 16-element chunks per lane: 2048 elements per warp
template <int FMT>
__global__ void __launch_bounds__(256) k_tc_prep_rows(const __grid_constant__ GemvParams p, uint8_t* xq,
                                                      int32_t* xshift, int mp, int np, int rows, int S) {
  __shared__ float s_part[2][8];  // per warp: sum of squares, maximum
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rl = warp / S, sec = warp % S;
  const int m = blockIdx.x * (8 / S) + rl;  // token (padded to whole token tiles)
  const int K = p.k;
  const size_t kb_bytes = static_cast<size_t>(np) * 128;
  constexpr int CPE = tc_bf16_operand(FMT) ? 2 : 1;  // 16-byte output chunks per 16 elements and term
  const bool live = m < rows;
  uint8_t* xt = xq + static_cast<size_t>(live ? m / mp : 0) * (K * (tc_bf16_operand(FMT) ? 2 : 1) / 128) * kb_bytes;
  const int ml = m % mp;
  auto off = [&](int n, int c) -> size_t {
    return static_cast<size_t>(c >> 3) * kb_bytes + static_cast<size_t>(n >> 3) * 1024 + (c & 7) * 128 + (n & 7) * 16;
  };
  auto chunk = [&](int j) { return sec * 32 * kRowsChunks + lane + 32 * j; };  // 16-element chunk index
  pdl_wait();
  pdl_launch();
  const bool pad_row = live && m < p.m && p.row_len && (m % p.row_T) >= p.row_len[p.row_b0 + m / p.row_T];
  const bool zero = live && (m >= p.m || pad_row);  // past the tokens, or a prompt's padding
  const bool work = live && !zero;
  const bool embed = p.pro == PRO_EMBED;
  uint4 raw[kRowsChunks][2];
  if (work) {
    const uint16_t* src;
    if (embed) {
      int64_t id = p.ids[m];
      id = id < 0 ? 0 : (id >= p.embed_rows ? p.embed_rows - 1 : id);  // never read outside the table
      src = p.embed + static_cast<size_t>(id) * K;
    } else {
      src = p.x + static_cast<size_t>(m) * K;
    }
#pragma unroll
    for (int j = 0; j < kRowsChunks; ++j) {
      raw[j][0] = *reinterpret_cast<const uint4*>(src + chunk(j) * 16);
      raw[j][1] = *reinterpret_cast<const uint4*>(src + chunk(j) * 16 + 8);
    }
  }
  // the 16 input values of chunk j (embedding rows: embed_tokens(ids) * 12, llm_mega.py:514)
  auto in16 = [&](int j, float* f) {
    unpack8(raw[j][0], f);
    unpack8(raw[j][1], f + 8);
    if (embed)
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = bf(f[e] * p.emb_mult);
  };
  // a row's total of per-warp values over its S sections (section order)
  auto row_total = [&](float v, int slot, bool is_max) {
    if (S == 1) return v;
    if (lane == 0) s_part[slot][warp] = v;
    __syncthreads();
    float t = 0.f;  // maxima are of magnitudes
    for (int q = 0; q < S; ++q) t = is_max ? fmaxf(t, s_part[slot][rl * S + q]) : t + s_part[slot][rl * S + q];
    return t;
  };
  float rstd = 0.f;
  if (p.pro != PRO_NONE) {  // RMSNorm statistics (modeling_granite.py:192-197)
    float ss = 0.f;
    if (work)
#pragma unroll
      for (int j = 0; j < kRowsChunks; ++j) {
        float f[16];
        in16(j, f);
        if (embed && p.hidden_out) {  // the residual stream of layer 0
          uint4* ho = reinterpret_cast<uint4*>(p.hidden_out + static_cast<size_t>(m) * K + chunk(j) * 16);
          ho[0] = pack8(f);
          ho[1] = pack8(f + 8);
        }
#pragma unroll
        for (int e = 0; e < 16; ++e) ss += f[e] * f[e];
      }
    ss = row_total(warp_sum(ss), 0, false);
    rstd = 1.f / sqrtf(ss / static_cast<float>(K) + p.eps);
  }
  // prologue output of chunk j: weight * bf16(x * rstd), or the input
  auto values16 = [&](int j, float* f) {
    in16(j, f);
    if (p.pro != PRO_NONE) {
      float wn[16];
      unpack8(__ldg(reinterpret_cast<const uint4*>(p.norm_w + chunk(j) * 16)), wn);
      unpack8(__ldg(reinterpret_cast<const uint4*>(p.norm_w + chunk(j) * 16 + 8)), wn + 8);
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = bf(wn[e] * bf(f[e] * rstd));
    }
  };
  if constexpr (tc_bf16_operand(FMT)) {
    if (work)
#pragma unroll
      for (int j = 0; j < kRowsChunks; ++j) {
        float f[16];
        values16(j, f);
        *reinterpret_cast<uint4*>(xt + off(ml, 2 * chunk(j))) = pack8(f);
        *reinterpret_cast<uint4*>(xt + off(ml, 2 * chunk(j) + 1)) = pack8(f + 8);
      }
  } else {
    float am = 0.f;
    if (work)
#pragma unroll
      for (int j = 0; j < kRowsChunks; ++j) {
        float f[16];
        values16(j, f);
#pragma unroll
        for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(f[e]));
      }
    am = row_total(warp_max(am), 1, true);
    const int shift = tc_fp8_shift(am);  // max |x| 2^shift in [128, 256)
    if (work) {
      if (sec == 0 && lane == 0) xshift[m] = shift;
#pragma unroll
      for (int j = 0; j < kRowsChunks; ++j) {
        float f[16];
        values16(j, f);
        uint4 w0, w1;
        e4m3_split16(f, shift, w0, w1);
        *reinterpret_cast<uint4*>(xt + off(ml, chunk(j))) = w0;
        *reinterpret_cast<uint4*>(xt + off(mp + ml, chunk(j))) = w1;
      }
    }
  }
  if (zero) {
#pragma unroll
    for (int j = 0; j < kRowsChunks; ++j)
#pragma unroll
      for (int e = 0; e < CPE; ++e) {
        *reinterpret_cast<uint4*>(xt + off(ml, CPE * chunk(j) + e)) = make_uint4(0, 0, 0, 0);
        if (FMT == SB_FMT_FP8) *reinterpret_cast<uint4*>(xt + off(mp + ml, chunk(j))) = make_uint4(0, 0, 0, 0);
      }
    if (FMT == SB_FMT_FP8 && sec == 0 && lane == 0) xshift[m] = 0;
  }
}

// One CTA per (padded) token row; the row is read once into registers (16
// consecutive elements per thread and chunk), then RMSNorm statistics, the
// power-of-two scale and the e4m3 split are all computed from registers.
// Rows >= m are written as zeros.
constexpr int kPrepCtaThreads = 256;
constexpr int kPrepChunks = 4;  // 16-element chunks per thread: K <= 16384

template <int FMT>
__global__ void __launch_bounds__(kPrepCtaThreads) k_tc_prep_cta(const __grid_constant__ GemvParams p, uint8_t* xq,
                                                           int32_t* xshift, int mp, int np) {
  __shared__ float s_red[kPrepCtaThreads / 32];
  const int m = blockIdx.x, tid = threadIdx.x, K = p.k;  // m: token (padded to whole token tiles)
  const int n16 = K / 16;
  const size_t kb_bytes = static_cast<size_t>(np) * 128;
  // token tile m / mp holds rows mp * tile .. of the operand, each tile [kb][np/8][8][8][16 B]
  uint8_t* xt = xq + static_cast<size_t>(m / mp) * (K * (tc_bf16_operand(FMT) ? 2 : 1) / 128) * kb_bytes;
  const int ml = m % mp;  // row of the token within its tile
  auto off = [&](int n, int c) -> size_t {  // 16-byte chunk c (along K bytes) of B-operand row n
    return static_cast<size_t>(c >> 3) * kb_bytes + static_cast<size_t>(n >> 3) * 1024 + (c & 7) * 128 + (n & 7) * 16;
  };
  constexpr int CPE = tc_bf16_operand(FMT) ? 2 : 1;  // 16-byte output chunks per 16 elements and term
  uint4 nw[kPrepChunks][2];  // RMSNorm weights: constant, read before waiting for the previous kernel
  if (p.pro != PRO_NONE && m < p.m)
#pragma unroll
    for (int j = 0; j < kPrepChunks; ++j) {
      const int c16 = tid + j * kPrepCtaThreads;
      if (c16 < n16) {
        nw[j][0] = __ldg(reinterpret_cast<const uint4*>(p.norm_w + c16 * 16));
        nw[j][1] = __ldg(reinterpret_cast<const uint4*>(p.norm_w + c16 * 16 + 8));
      }
    }
  pdl_wait();
  pdl_launch();
  const bool pad_row = m < p.m && p.row_len && (m % p.row_T) >= p.row_len[p.row_b0 + m / p.row_T];
  if (m >= p.m || pad_row) {  // past the tokens, or a prompt's padding: zero operand rows
    for (int c = tid; c < n16 * CPE; c += kPrepCtaThreads) {
      *reinterpret_cast<uint4*>(xt + off(ml, c)) = make_uint4(0, 0, 0, 0);
      if (FMT == SB_FMT_FP8) *reinterpret_cast<uint4*>(xt + off(mp + ml, c)) = make_uint4(0, 0, 0, 0);
    }
    if (FMT == SB_FMT_FP8 && tid == 0) xshift[m] = 0;
    return;
  }
  const bool embed = p.pro == PRO_EMBED;
  const uint16_t* src;
  if (embed) {
    int64_t id = p.ids[m];
    id = id < 0 ? 0 : (id >= p.embed_rows ? p.embed_rows - 1 : id);  // never read outside the table
    src = p.embed + static_cast<size_t>(id) * K;
  } else {
    src = p.x + static_cast<size_t>(m) * K;
  }
  float f[kPrepChunks][16];
#pragma unroll
  for (int j = 0; j < kPrepChunks; ++j) {
    const int c16 = tid + j * kPrepCtaThreads;
    if (c16 < n16) {
      unpack8(*reinterpret_cast<const uint4*>(src + c16 * 16), f[j]);
      unpack8(*reinterpret_cast<const uint4*>(src + c16 * 16 + 8), f[j] + 8);
      if (embed) {  // embed_tokens(ids) * 12 (llm_mega.py:514): the residual stream of layer 0
#pragma unroll
        for (int e = 0; e < 16; ++e) f[j][e] = bf(f[j][e] * p.emb_mult);
        if (p.hidden_out) {
          uint4* ho = reinterpret_cast<uint4*>(p.hidden_out + static_cast<size_t>(m) * K + c16 * 16);
          ho[0] = pack8(f[j]);
          ho[1] = pack8(f[j] + 8);
        }
      }
    }
  }
  if (p.pro != PRO_NONE) {  // weight * bf16(x * rstd)  (modeling_granite.py:192-197)
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kPrepChunks; ++j)
      if (tid + j * kPrepCtaThreads < n16)
#pragma unroll
        for (int e = 0; e < 16; ++e) ss += f[j][e] * f[j][e];
    ss = block_sum256(ss, s_red);
    const float rstd = 1.f / sqrtf(ss / static_cast<float>(K) + p.eps);
#pragma unroll
    for (int j = 0; j < kPrepChunks; ++j) {
      const int c16 = tid + j * kPrepCtaThreads;
      if (c16 < n16) {
        float wn[16];
        unpack8(nw[j][0], wn);
        unpack8(nw[j][1], wn + 8);
#pragma unroll
        for (int e = 0; e < 16; ++e) f[j][e] = bf(wn[e] * bf(f[j][e] * rstd));
      }
    }
  }
  if constexpr (tc_bf16_operand(FMT)) {
#pragma unroll
    for (int j = 0; j < kPrepChunks; ++j) {
      const int c16 = tid + j * kPrepCtaThreads;
      if (c16 < n16) {
        *reinterpret_cast<uint4*>(xt + off(ml, 2 * c16)) = pack8(f[j]);
        *reinterpret_cast<uint4*>(xt + off(ml, 2 * c16 + 1)) = pack8(f[j] + 8);
      }
    }
  } else {
    float am = 0.f;
#pragma unroll
    for (int j = 0; j < kPrepChunks; ++j)
      if (tid + j * kPrepCtaThreads < n16)
#pragma unroll
        for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(f[j][e]));
    am = block_max256(am, s_red);
    int e2 = 0;
    if (am > 0.f) frexpf(am, &e2);
    const int shift = 8 - e2;  // max |x| 2^shift in [128, 256)
    if (tid == 0) xshift[m] = shift;
#pragma unroll
    for (int j = 0; j < kPrepChunks; ++j) {
      const int c16 = tid + j * kPrepCtaThreads;
      if (c16 < n16) {
        uint4 w0, w1;
        e4m3_split16(f[j], shift, w0, w1);
        *reinterpret_cast<uint4*>(xt + off(ml, c16)) = w0;
        *reinterpret_cast<uint4*>(xt + off(mp + ml, c16)) = w1;
      }
    }
  }
}

// ---- the GEMM ----------------------------------------------------------------------
// NEPI epilogue warps: 8 with two CTAs per SM, 16 with one
// OPB: the B operand is block-scaled (written by the preceding GEMM's epilogue;
// fp8 only), the MMA kind::mxf8f6f4 with UE8M0 scales
template <int FMT, int EPI, int NEPI, int OPB>
__global__ void __launch_bounds__((NEPI + 2) * 32, NEPI == kTcEpiWarps ? 2 : 1)
    k_tc_gemm(const __grid_constant__ GemvParams p, const __grid_constant__ TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nepi = NEPI;
  auto epi_bar = [&]() { asm volatile("bar.sync 1, %0;" ::"n"(NEPI * 32) : "memory"); };
  const int M = p.m;
  const TcLayout L = tc_layout(a.np, a.stages, M, a.split, NEPI, OPB != 0);
  uint8_t* ring = smem;
  float* part = reinterpret_cast<float*>(smem + L.part);  // split: inbox [src rank][row][ms]
  const int ms = tc_inbox_stride(M);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint64_t* empty = full + a.stages;
  uint64_t* acc_full = empty + a.stages;  // [2]: double-buffered accumulator
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(smem + L.tmem);
  int* s_flag = reinterpret_cast<int*>(smem + L.flag);
  int* s_best = reinterpret_cast<int*>(smem + L.best);
  float* s_bval = reinterpret_cast<float*>(smem + L.bval);
  int* s_shift = reinterpret_cast<int*>(smem + L.shift);
  float* wb_val = reinterpret_cast<float*>(smem + L.wbv);
  int* wb_idx = reinterpret_cast<int*>(smem + L.wbi);
  // QKV: per token of the current token tile its RoPE position, stream and
  // position in the stream, plus the cache slot of position 0 (tc_epi's
  // tokpos layout; the argmax scratch is unused by this epilogue)
  int* s_tokpos = reinterpret_cast<int*>(wb_val);
  const int* tokpos = EPI == EPI_QKV ? s_tokpos : nullptr;
  int32_t* err = p.ctrl ? p.ctrl + SB_CTRL_ERR : nullptr;

  const int S = a.split;
  const int q = S > 1 ? static_cast<int>(cg::this_cluster().block_rank()) : 0;
  const int cid = blockIdx.x / S, ncl = gridDim.x / S;
  const int kb0 = q * a.kb / S, kb1 = (q + 1) * a.kb / S, nk = kb1 - kb0;
  // token tiles that hold at least one real row (prefill of right-padded
  // prompts: tiles entirely in padding are skipped by every role alike)
  int* s_live = reinterpret_cast<int*>(smem + L.live);
  if (tid == 0) {
    int n = 0;
    for (int tt = 0; tt < a.mtiles && tt < 64; ++tt) {
      bool real = !p.row_len;
      const int r0 = tt * a.mp, r1 = min(r0 + a.mp, M);
      for (int r = r0; r < r1 && !real;) {  // one check per stream overlapping the tile
        const int b = r / p.row_T, pos = r % p.row_T;
        if (pos < p.row_len[p.row_b0 + b]) real = true;
        r = (b + 1) * p.row_T;
      }
      if (real) s_live[1 + n++] = tt;
    }
    s_live[0] = n;
  }
  __syncthreads();
  const int nlive = s_live[0];
  // work items (weight tile, live token tile), token tiles inner so that the
  // CTAs working at the same time share weight tiles (L2 hits)
  const int items = a.tiles * nlive;
  const int my_tiles = cid < items ? (items - cid + ncl - 1) / ncl : 0;
  const uint32_t a_bytes = 16384u, b_bytes = static_cast<uint32_t>(a.np) * 128u + (OPB ? 512u : 0u);
  // CTAs start their K blocks at different offsets so that they do not all read
  // the same activation block from L2 at the same time
  const int rot = cid % nk;
  const uint32_t half_cols = static_cast<uint32_t>(a.ncols) / 2;  // accumulator buffer stride

  constexpr int kProd = nepi, kMma = nepi + 1;  // warp roles
  if (warp == kProd && lane == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b2 = 0; b2 < 2; ++b2) {
      mbar_init(acc_full + b2, 1);
      mbar_init(acc_empty + b2, nepi * 32);
    }
    mbar_fence_init();
  }
  if (warp == kMma) tmem_alloc(s_tmem, static_cast<uint32_t>(OPB ? a.tmem_cols : a.ncols));
  if constexpr (OPB != 0) {  // the weight's block scales: all 1.0 (its row scales come in the epilogue)
    if (tid < 128) reinterpret_cast<uint32_t*>(smem + L.sfa)[tid] = 0x7F7F7F7Fu;
    tc_fence_proxy_smem();  // generic writes read by tcgen05.cp
  }
  if constexpr (EPI == EPI_ARGMAX)
    for (int i = tid; i < (nepi + 2) * 128; i += blockDim.x) {
      wb_val[i] = -INFINITY;
      wb_idx[i] = 0x7fffffff;
    }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == kProd) {
    // ---- producer ----
    if (lane == 0) {
      const int total = my_tiles * nk;
      auto kb_of = [&](int it) { return kb0 + (it % nk + rot) % nk; };
      auto a_src = [&](int it) {
        const int t = (cid + (it / nk) * ncl) / nlive;
        return a.wt + (static_cast<size_t>(t) * a.kb + kb_of(it)) * 16384;
      };
      auto b_src = [&](int it) {
        const int tt = s_live[1 + (cid + (it / nk) * ncl) % nlive];
        return a.xq + (static_cast<size_t>(tt) * a.kb + kb_of(it)) * b_bytes;
      };
      const int pre = total < a.stages ? total : a.stages;
      for (int it = 0; it < pre; ++it) {  // weights do not depend on the previous kernel
        mbar_expect_tx(full + it, a_bytes + b_bytes);
        bulk_g2s(ring + it * L.stage_bytes, a_src(it), a_bytes, full + it);
      }
      pdl_wait();
      for (int it = 0; it < pre; ++it) bulk_g2s(ring + it * L.stage_bytes + 16384, b_src(it), b_bytes, full + it);
      for (int it = pre; it < total; ++it) {
        const int s = it % a.stages;
        wait_bounded(empty + s, static_cast<uint32_t>((it / a.stages - 1) & 1), err);
        mbar_expect_tx(full + s, a_bytes + b_bytes);
        bulk_g2s(ring + s * L.stage_bytes, a_src(it), a_bytes, full + s);
        bulk_g2s(ring + s * L.stage_bytes + 16384, b_src(it), b_bytes, full + s);
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
      if constexpr (OPB != 0) tc_cp_scales(tmem + static_cast<uint32_t>(a.sfa_col), sdesc(su32(smem + L.sfa), 0u, 128u));
      int it = 0;
      for (int tc = 0; tc < my_tiles; ++tc) {
        const int buf = tc & 1;
        if (tc >= 2) wait_bounded(acc_empty + buf, static_cast<uint32_t>((tc / 2 - 1) & 1), err);
        tc_fence_after();
        const uint32_t dacc = tmem + buf * half_cols;
        for (int j = 0; j < nk; ++j, ++it) {
          const int s = it % a.stages;
          wait_bounded(full + s, static_cast<uint32_t>((it / a.stages) & 1), err);
          tc_fence_after();
          const uint32_t sa = su32(ring + s * L.stage_bytes), sbb = sa + 16384u;
          if constexpr (OPB != 0) {
            // this stage's B scales into its own four TMEM columns (no copy
            // rewrites columns that an issued MMA may still read), then one
            // MMA per 32-element block, each reading byte kk of the scale words
            const uint32_t tsfb = tmem + static_cast<uint32_t>(a.sfb_col + 4 * s);
            tc_cp_scales(tsfb, sdesc(sbb + static_cast<uint32_t>(a.np) * 128u, 0u, 128u));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_mx8(dacc, sdesc(sa + kk * 256u, 128u, 1024u), sdesc(sbb + kk * 256u, 128u, 1024u),
                         a.idesc | (static_cast<uint32_t>(kk) << 4) | (static_cast<uint32_t>(kk) << 29),
                         tmem + static_cast<uint32_t>(a.sfa_col), tsfb, (j > 0 || kk > 0) ? 1u : 0u);
          } else {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma<FMT>(dacc, sdesc(sa + kk * 256u, 128u, 1024u), sdesc(sbb + kk * 256u, 128u, 1024u), a.idesc,
                          (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(empty + s);  // the stage is free once these MMAs have read it
        }
        tc_commit(acc_full + buf);
      }
    }
    __syncwarp();
  } else {
    // ---- epilogue warps 0-7: warp w reads TMEM lanes 32 (w % 4).. (tile rows) and
    // the 8-token chunks h, h + 2, ... with h = w / 4 ----
    pdl_wait();
    pdl_launch();
    // bring the epilogue's global inputs into L1 while the main loop runs: the
    // weight row scales and residual rows of the CTA's first tile (or its
    // rank's rows of the shared tile), and the RoPE rows at each token's position
    if ((FMT == SB_FMT_FP8 || FMT == SB_FMT_INT8) && my_tiles > 0 && tid < 4) {
      const int r = (cid / nlive) * 128 + tid * 32;  // 32 fp32 scales = one 128-byte line
      if (r < p.n) asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const float*>(p.scale) + r));
    }
    if (a.mtiles > 1) {
      // prefill token tiles: no prefetch
    } else if constexpr (EPI == EPI_RESID) {
      const int rp0 = tc_rows_per_rank(S);
      const int ra = cid * 128 + (S > 1 ? q * rp0 : 0), nr = S > 1 ? rp0 : 128;
      const int rb = min(ra + nr, p.n);
      const int nseg = (rb - ra + 63) / 64;  // 128-byte lines of bf16 rows
      for (int i = tid; i < M * nseg; i += nepi * 32)
        if (ra < rb)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(p.y + static_cast<size_t>(i / nseg) * p.n + ra + (i % nseg) * 64));
    }
    float* s_unscale = reinterpret_cast<float*>(s_shift);  // 2^-shift per token of the tile: exact
    constexpr int nh = nepi >> 2;
    const int lq = warp & 3, h = warp >> 2;  // lane quarter; token chunk offset (stride nh)
    const int lrow = lq * 32 + lane;
    const int rp = tc_rows_per_rank(S);
    float* s_stage = reinterpret_cast<float*>(wb_val);  // decode chain: [tokens][64 activations]
    for (int tc = 0; tc < my_tiles; ++tc) {
      const int item = cid + tc * ncl, buf = tc & 1;
      const int t = item / nlive, tok0 = s_live[1 + item % nlive] * a.mp;
      const int Mt = M - tok0 < a.mp ? M - tok0 : a.mp;  // tokens of this tile
      if (FMT == SB_FMT_FP8 || EPI == EPI_QKV) {
        epi_bar();  // every warp is done with the previous tile's scales / token table
        if constexpr (OPB != 0) {
          // the block scales are in the MMA; what remains is the consumer's
          // RMSNorm 1 / rms from the producer's sums of squares (fixed order;
          // one warp per token, up to four tokens per warp, every load in
          // flight at once)
          if (p.ssq_in) {
            const int ns = p.k >> 5;  // slices of 32 rows per token
            float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = warp + u * nepi;
              if (i < Mt)
                for (int j = lane; j < ns; j += 32) ss[u] += p.ssq_in[static_cast<size_t>(tok0 + i) * ns + j];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = warp + u * nepi;
              const float t = warp_sum(ss[u]);
              if (lane == 0 && i < Mt) s_unscale[i] = 1.f / sqrtf(t / static_cast<float>(p.k) + p.eps);
            }
          } else {
            for (int i = tid; i < Mt; i += nepi * 32) s_unscale[i] = 1.f;
          }
        } else if (FMT == SB_FMT_FP8) {
          const int32_t* xs = a.xshift + (a.rank_shift ? q * a.mp : 0);  // this rank's K range has its own scale
          for (int i = tid; i < Mt; i += nepi * 32) s_unscale[i] = ldexpf(1.f, -xs[tok0 + i]);
        }
        if constexpr (EPI == EPI_QKV) {
          // the tile's tokens, once (the epilogue would otherwise chain three
          // dependent global loads per call: control block, rope_off, tables)
          const int slot_base = p.ctrl[SB_CTRL_SLOT];
          for (int i = tid; i < Mt; i += nepi * 32) {
            const int m = tok0 + i, b = m / p.m_per, mi = m % p.m_per;
            int pos = slot_base + mi - (p.rope_off ? p.rope_off[b] : 0);
            pos = pos < 0 ? 0 : (pos >= p.rope_max ? p.rope_max - 1 : pos);
            s_tokpos[i] = pos;
            s_tokpos[129 + i] = b;
            s_tokpos[257 + i] = mi;
            asm volatile("prefetch.global.L1 [%0];" ::"l"(p.cos_tab + static_cast<size_t>(pos) * 64));
            asm volatile("prefetch.global.L1 [%0];" ::"l"(p.sin_tab + static_cast<size_t>(pos) * 64));
          }
          if (tid == 0) s_tokpos[128] = slot_base;
        }
        epi_bar();
      }
      const uint32_t taddr = tmem + buf * half_cols + (static_cast<uint32_t>(lq * 32) << 16);
      wait_bounded(acc_full + buf, static_cast<uint32_t>((tc / 2) & 1), err);
      tc_fence_after();
      for (int m0 = h * 8; m0 < Mt; m0 += 8 * nh) {
        // 8 tokens of this lane's row: D0 (and D1 for the fp8 split) columns
        uint32_t d0[8], d1[8];
        tmem_ld8(taddr + m0, d0);
        if (FMT == SB_FMT_FP8) tmem_ld8(taddr + a.mp + m0, d1);
        tmem_wait_ld();
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[i] = __uint_as_float(d0[i]);
          if (FMT == SB_FMT_FP8) {
            const int m = m0 + i < Mt ? m0 + i : Mt - 1;
            v[i] = fmaf(__uint_as_float(d1[i]), 0.0625f, v[i]) * s_unscale[m];  // (D0 + D1/16) 2^-s
          }
        }
        if (S == 1) {
          const int row = t * 128 + lrow;
          tc_epi<FMT, 8, EPI>(p, row, row < p.n, v, m0, Mt, wb_val, wb_idx, warp, tok0, tokpos);
          if constexpr (EPI == EPI_SWIGLU) {
            // decode chain: stage the activations (even lanes) for the down
            // projection's operand, written by the whole epilogue below
            if (p.nx_op && !(lane & 1) && row < p.n)
#pragma unroll
              for (int i = 0; i < 8; ++i)
                if (m0 + i < Mt) s_stage[(m0 + i) * 64 + (lrow >> 1)] = v[i];
          }
        } else {
          // push this K partial to the rank that finishes the row (16-byte DSMEM stores)
          float* dst = cg::this_cluster().map_shared_rank(part, lrow / rp) + (q * rp + lrow % rp) * ms + m0;
          reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
          reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty + buf);  // the MMA warp may overwrite this accumulator
      if constexpr (EPI == EPI_SWIGLU) {
        if (S == 1 && p.nx_op) {  // the tile's 64 activations of every token -> the down projection's operand
          epi_bar();
          tc_bs_write_tile(p.nx_op, p.nx_np, p.nx_mp, tok0, t * 64, 64, s_stage, Mt, nullptr, nullptr, 0, tid, nepi * 32);
        }
      }
    }
  }

  if (S > 1) {  // one tile per cluster: sum the pushed K partials in rank order, then the epilogue
    cg::this_cluster().sync();  // every partial has landed in its owner's inbox
    const int rp = tc_rows_per_rank(S), r0 = q * rp;
    const int nr = r0 >= 128 ? 0 : (r0 + rp > 128 ? 128 - r0 : rp);
    // items of (32-row group, 4 tokens) over all warps; one float4 (16-byte,
    // conflict-free) inbox read per source rank
    const int nw = blockDim.x >> 5, ngrp = (nr + 31) / 32, nch = (M + 3) / 4;
    for (int item = warp; item < ngrp * nch; item += nw) {
      const int rg = item / nch, m0 = (item % nch) * 4;
      const int lr = rg * 32 + lane;
      const bool ok = lr < nr;
      if constexpr (EPI == EPI_RESID)  // decode chain: the next RMSNorm weight of these 32 rows, into L1 now
        if (p.nx_op && lane == 0)
          asm volatile("prefetch.global.L1 [%0];" ::"l"(p.nx_g + cid * 128 + r0 + rg * 32));
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok)
        for (int c = 0; c < S; ++c) {
          const float4 x4 = *reinterpret_cast<const float4*>(part + (c * rp + lr) * ms + m0);
          v[0] += x4.x;
          v[1] += x4.y;
          v[2] += x4.z;
          v[3] += x4.w;
        }
      const int row = cid * 128 + r0 + lr;
      tc_epi<FMT, 4, EPI>(p, row, ok && row < p.n, v, m0, M, wb_val, wb_idx, warp, 0, tokpos);
      if constexpr (EPI == EPI_RESID) {
        if (p.nx_op) {
          // decode chain: this item's 32 new rows of 4 tokens, times the next
          // RMSNorm weight, as the next projection's operand (whole 32-element
          // blocks: no other warp involved), plus their sums of squares
          float* sv = reinterpret_cast<float*>(wb_val) + warp * 128;  // [4 tokens][32 rows]
#pragma unroll
          for (int i = 0; i < 4; ++i) sv[i * 32 + lane] = ok ? v[i] : 0.f;
          __syncwarp();
          const int nt = M - m0 < 4 ? M - m0 : 4;
          tc_bs_write_tile(p.nx_op, p.nx_np, p.nx_mp, m0, cid * 128 + r0 + rg * 32, 32, sv, nt, p.nx_g, p.nx_ssq,
                           p.n >> 5, lane, 32);
          __syncwarp();
        }
      }
    }
  }
  if constexpr (EPI == EPI_ARGMAX) {  // combine the warps' running bests (order-independent total order)
    __syncthreads();
    for (int m = tid; m < M; m += blockDim.x) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int w = 0; w < nepi + 2; ++w)
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
    tmem_dealloc(tmem, static_cast<uint32_t>(OPB ? a.tmem_cols : a.ncols));
  }
}

// ---- host side ------------------------------------------------------------------
static const int kSMs = 148;
static const size_t kTcSmem = 220 * 1024;
static const int kTcShiftRanks = 8;  // the widest K split (clusters of 8)

static int elem_bytes(int fmt) { return tc_bf16_operand(fmt) ? 2 : 1; }
static int pad_rows(int fmt, int m) { return tc_bf16_operand(fmt) ? (m + 15) / 16 * 16 : (m + 7) / 8 * 8; }

// token rows above 128 are processed in tiles of 128 (one launch)
static int tile_rows(int fmt, int m) { return m > 128 ? 128 : pad_rows(fmt, m); }

size_t tc_shift_offset(int fmt, int k, int m) {
  const int mp = tile_rows(fmt, m), mtiles = (m + mp - 1) / mp;
  const int np = fmt == SB_FMT_FP8 ? 2 * mp : mp;
  return static_cast<size_t>(mtiles) * np * k * elem_bytes(fmt);
}

size_t tc_operand_bytes(int fmt, int k, int m) {
  if (!tc_format(fmt) || m < 1) return 0;
  const int mp = tile_rows(fmt, m), mtiles = (m + mp - 1) / mp;
  const int np = fmt == SB_FMT_FP8 ? 2 * mp : mp;
  // shifts: one row per token tile, or one per K-split rank (operand written per rank)
  const int srows = mtiles > kTcShiftRanks ? mtiles : kTcShiftRanks;
  return static_cast<size_t>(mtiles) * np * k * elem_bytes(fmt) + static_cast<size_t>(srows) * mp * 4;
}

static int tc_ctas_per_sm_max() { return 2; }

static const size_t kTcSmemTwo = 110 * 1024;  // two CTAs per SM

// Plan for per_sm CTAs per SM.  Two CTAs per SM (decode / verify: one token
// tile, many weight tiles) halve the ring and the TMEM of each but run two
// MMA-issuing threads per SM, which is what bounds the streaming of a CTA at
// these shapes (four MMAs per stage, issue latency rather than tensor-pipe
// time).
// bs: block-scaled operand (one CTA per SM; TMEM also holds the scales);
// max_split: the widest K split allowed
static bool tc_plan_for(int fmt, int n, int k, int m, int per_sm, TcPlan& pl, bool bs = false, int max_split = 8) {
  if (bs && per_sm != 1) return false;
  const int eb = elem_bytes(fmt);
  pl.mp = tile_rows(fmt, m);
  pl.mtiles = (m + pl.mp - 1) / pl.mp;
  pl.np = fmt == SB_FMT_FP8 ? 2 * pl.mp : pl.mp;
  if (pl.np < 16 || pl.np > 256) return false;
  if (pl.mtiles > 64) return false;  // the GEMM keeps a list of at most 64 token tiles
  if (per_sm > 1 && pl.mtiles > 1) return false;
  pl.tiles = (n + 127) / 128;
  pl.kb = k * eb / 128;
  const int slots = kSMs * per_sm;
  // measured at 48 rows: two CTAs per SM pay off for persistent plans over
  // hundreds of tiles (lm_head 88.8 -> 73.1 us) but not with K split over
  // clusters of 8 (q/k/v 14.9 -> 16.9, o 9.7 -> 10.5 us; gate/up, down even)
  if (per_sm > 1 && pl.tiles * 4 < slots * 3) return false;
  if (pl.mtiles > 1) {  // many token tiles (prefill): persistent over (weight tile, token tile)
    pl.split = 1;
    const int items = pl.tiles * pl.mtiles;
    pl.n_ctas = items < kSMs ? items : kSMs;
  } else if (pl.tiles * 4 >= slots * 3) {  // enough tiles: persistent, no K split
    pl.split = 1;
    pl.n_ctas = pl.tiles < slots ? pl.tiles : slots;
  } else {
    // one CTA per SM: clusters of more than 4 CTAs of ~200 KiB do not all fit at once
    int s = slots / pl.tiles;
    int smax = per_sm > 1 ? 8 : 4;
    if (smax > max_split) smax = max_split;
    if (s > smax) s = smax;
    if (s > pl.kb) s = pl.kb;
    if (s < 1) s = 1;
    pl.split = s;
    pl.n_ctas = pl.tiles * s;
  }
  pl.ncols = 32;
  while (pl.ncols < 2 * pl.np) pl.ncols *= 2;  // two accumulator buffers
  pl.epi_warps = per_sm > 1 ? kTcEpiWarps : kTcMaxEpiWarps;  // (the layout below depends on it)
  if (per_sm > 1 && pl.ncols > 256) return false;
  const size_t budget = per_sm > 1 ? kTcSmemTwo : kTcSmem;
  pl.stages = 0;
  const int ml = m < pl.mp ? m : pl.mp;  // token rows of one tile
  pl.bs = bs ? 1 : 0;
  pl.tmem_cols = pl.ncols;
  for (int st = 8; st >= 2; --st)
    if (tc_layout(pl.np, st, ml, pl.split, pl.epi_warps, bs).total <= budget && (!bs || pl.ncols + 4 + 4 * st <= 512)) {
      pl.stages = st;
      break;
    }
  if (!pl.stages) return false;
  if (bs)  // the accumulators, then the weight's scales (4 columns) and 4 per stage for B's
    while (pl.tmem_cols < pl.ncols + 4 + 4 * pl.stages) pl.tmem_cols *= 2;
  pl.smem = tc_layout(pl.np, pl.stages, ml, pl.split, pl.epi_warps, bs).total;
  return true;
}

bool tc_plan(int fmt, int n, int k, int m, TcPlan& pl) {
  if (!tc_format(fmt) || m < 1 || n < 1) return false;
  const int eb = elem_bytes(fmt);
  if ((k * eb) % 128 != 0 || k > kPrepMaxK || k > 16 * kPrepCtaThreads * kPrepChunks) return false;
  if (tc_ctas_per_sm_max() >= 2 && tc_plan_for(fmt, n, k, m, 2, pl)) return true;
  return tc_plan_for(fmt, n, k, m, 1, pl);
}

template <int FMT, int EPI, int NEPI, int OPB = 0>
static int gemm_launch_n(const cudaLaunchConfig_t& cfg, const GemvParams& p, const TcArgs& a) {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<unsigned> configured{0};  // one bit per device
  if (!(configured.load(std::memory_order_relaxed) & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(k_tc_gemm<FMT, EPI, NEPI, OPB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kTcSmem));
    if (e != cudaSuccess) return e;
    configured.fetch_or(1u << dev, std::memory_order_relaxed);
  }
  return cudaLaunchKernelEx(&cfg, k_tc_gemm<FMT, EPI, NEPI, OPB>, p, a);
}

template <int FMT, int EPI>
static int gemm_launch(int epi_warps, const cudaLaunchConfig_t& cfg, const GemvParams& p, const TcArgs& a) {
  return epi_warps == kTcEpiWarps ? gemm_launch_n<FMT, EPI, kTcEpiWarps>(cfg, p, a)
                                  : gemm_launch_n<FMT, EPI, kTcMaxEpiWarps>(cfg, p, a);
}

template <int FMT>
static int tc_launch_t(const GemvParams& p0, const void* w_tc, void* operand, const TcPlan& pl, bool pdl,
                       cudaStream_t stream, bool operand_ready) {
  GemvParams p = p0;
  p.n_ctas = pl.n_ctas;
  uint8_t* xq = static_cast<uint8_t*>(operand);
  int32_t* xshift =
      reinterpret_cast<int32_t*>(xq + static_cast<size_t>(pl.mtiles) * pl.np * p.k * elem_bytes(FMT));

  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  const int rows = pl.mp * pl.mtiles;
  const bool per_warp = pl.mtiles > 1;
  // many rows: rows held in registers when K is 2048 x (1, 2, 4 or 8), else one warp per row
  const int S = p.k % (32 * 16 * kRowsChunks) == 0 ? p.k / (32 * 16 * kRowsChunks) : 0;
  const bool in_regs = per_warp && (S == 1 || S == 2 || S == 4 || S == 8);
  cfg.gridDim = dim3(in_regs ? (rows + 8 / S - 1) / (8 / S) : per_warp ? (rows + kPrepRows - 1) / kPrepRows : rows);
  cfg.blockDim = dim3(in_regs ? 256 : per_warp ? kPrepThreads : kPrepCtaThreads);
  cfg.stream = stream;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  if (!operand_ready) {  // else the preceding kernel wrote the operand (and, fp8, its per-rank shifts)
    note_launch();
    cudaError_t e =
        in_regs    ? cudaLaunchKernelEx(&cfg, k_tc_prep_rows<FMT>, p, xq, xshift, pl.mp, pl.np, rows, S)
        : per_warp ? cudaLaunchKernelEx(&cfg, k_tc_prep_warp<FMT>, p, xq, xshift, pl.mp, pl.np, rows)
                   : cudaLaunchKernelEx(&cfg, k_tc_prep_cta<FMT>, p, xq, xshift, pl.mp, pl.np);
    if (e != cudaSuccess) return e;
  }

  TcArgs a;
  a.wt = static_cast<const uint8_t*>(w_tc);
  a.xq = xq;
  a.xshift = xshift;
  // instruction descriptor: D f32, A/B K-major, A/B e4m3 (f8f6f4) or bf16 (f16), N, M = 128
  const uint32_t ab = tc_bf16_operand(FMT) ? 1u : 0u;
  a.idesc = (1u << 4) | (ab << 7) | (ab << 10) | (static_cast<uint32_t>(pl.np >> 3) << 17) | ((128u >> 4) << 24);
  a.mp = pl.mp;
  a.np = pl.np;
  a.tiles = pl.tiles;
  a.kb = pl.kb;
  a.split = pl.split;
  a.stages = pl.stages;
  a.ncols = pl.ncols;
  a.mtiles = pl.mtiles;
  a.rank_shift = operand_ready && FMT == SB_FMT_FP8 ? 1 : 0;
  cfg.gridDim = dim3(pl.n_ctas);
  cfg.blockDim = dim3((pl.epi_warps + 2) * 32);
  cfg.dynamicSmemBytes = pl.smem;
  int na = 0;
  if (pdl) at[na++] = at[0];
  if (pl.split > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = pl.split;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.numAttrs = na;
  note_launch();
  switch (p.epi) {
    case EPI_STORE: return gemm_launch<FMT, EPI_STORE>(pl.epi_warps, cfg, p, a);
    case EPI_QKV: return gemm_launch<FMT, EPI_QKV>(pl.epi_warps, cfg, p, a);
    case EPI_RESID: return gemm_launch<FMT, EPI_RESID>(pl.epi_warps, cfg, p, a);
    case EPI_SWIGLU: return gemm_launch<FMT, EPI_SWIGLU>(pl.epi_warps, cfg, p, a);
    case EPI_ARGMAX: return gemm_launch<FMT, EPI_ARGMAX>(pl.epi_warps, cfg, p, a);
  }
  return SB_ERR_ARG;
}

int tc_launch(const GemvParams& p, const void* w_tc, void* operand, const TcPlan& pl, int fmt, bool pdl,
              cudaStream_t stream, bool operand_ready) {
  switch (fmt) {
    case SB_FMT_BF16: return tc_launch_t<SB_FMT_BF16>(p, w_tc, operand, pl, pdl, stream, operand_ready);
    case SB_FMT_FP8: return tc_launch_t<SB_FMT_FP8>(p, w_tc, operand, pl, pdl, stream, operand_ready);
    case SB_FMT_INT8: return tc_launch_t<SB_FMT_INT8>(p, w_tc, operand, pl, pdl, stream, operand_ready);
    case SB_FMT_NVFP4: return tc_launch_t<SB_FMT_NVFP4>(p, w_tc, operand, pl, pdl, stream, operand_ready);
  }
  return SB_ERR_ARG;
}

}  // namespace sb

namespace sb {

bool tc_plan_bs(int n, int k, int m, int max_split, TcPlan& pl) {
  if (m < 9 || m > 64 || n < 1 || k % 128 != 0) return false;
  return tc_plan_for(SB_FMT_FP8, n, k, m, 1, pl, true, max_split) && pl.mtiles == 1 &&
         pl.epi_warps == kTcMaxEpiWarps;
}

size_t tc_bs_operand_bytes(int k, int m) {
  const int np = 2 * pad_rows(SB_FMT_FP8, m);
  return static_cast<size_t>(k / 128) * tc_bs_block_bytes(np);
}

int tc_launch_bs(const GemvParams& p0, const void* w_tc, const void* operand, const TcPlan& pl, bool pdl,
                 cudaStream_t stream) {
  if (!pl.bs || pl.epi_warps != kTcMaxEpiWarps || pl.mtiles != 1) return SB_ERR_ARG;
  GemvParams p = p0;
  p.n_ctas = pl.n_ctas;
  TcArgs a;
  memset(&a, 0, sizeof(a));
  a.wt = static_cast<const uint8_t*>(w_tc);
  a.xq = static_cast<const uint8_t*>(operand);
  // instruction descriptor (block-scaled): A/B e4m3 (0), K-major, UE8M0 scales
  // (bit 23), N, M = 128; the scale ids (bits 4-5, 29-30) are set per MMA
  a.idesc = (1u << 23) | (static_cast<uint32_t>(pl.np >> 3) << 17) | ((128u >> 4) << 24);
  a.mp = pl.mp;
  a.np = pl.np;
  a.tiles = pl.tiles;
  a.kb = pl.kb;
  a.split = pl.split;
  a.stages = pl.stages;
  a.ncols = pl.ncols;
  a.mtiles = pl.mtiles;
  a.tmem_cols = pl.tmem_cols;
  a.sfa_col = pl.ncols;
  a.sfb_col = pl.ncols + 4;
  cudaLaunchAttribute at[2];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_ctas);
  cfg.blockDim = dim3((pl.epi_warps + 2) * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cfg.attrs = at;
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
  cfg.numAttrs = na;
  note_launch();
  switch (p.epi) {
    case EPI_QKV: return gemm_launch_n<SB_FMT_FP8, EPI_QKV, kTcMaxEpiWarps, 1>(cfg, p, a);
    case EPI_RESID: return gemm_launch_n<SB_FMT_FP8, EPI_RESID, kTcMaxEpiWarps, 1>(cfg, p, a);
    case EPI_SWIGLU: return gemm_launch_n<SB_FMT_FP8, EPI_SWIGLU, kTcMaxEpiWarps, 1>(cfg, p, a);
  }
  return SB_ERR_ARG;
}

}  // namespace sb
