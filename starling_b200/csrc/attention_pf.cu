// Prefill attention over right-padded prompts, sm_100a.
//
// The reference computes the prompt's attention with the eager HF path
// (llm_mega.py:176-202 -> modeling_granite.py:89-112): scores over every key,
// additive causal mask, fp32 softmax cast to bf16, probs @ V.  The decode
// kernel (attention.cu) keeps a block's whole score row in shared memory,
// which limits it to query blocks of 8 positions at prompt lengths of ~900,
// so each stream's K/V would be read by T/8 CTAs.  Here one CTA takes
// 128 query rows -- 128 / G positions x the G query heads of one KV head --
// and keeps no scores: it reads the block's keys twice.
//  * pass 1: S = Q K^T tile by tile (64 keys), score = bf16(bf16(q.k) * scale),
//    causal and prompt-length mask, row max and the fp32 exp-sum (rescaled
//    when the max grows);
//  * pass 2: the same scores again, p = bf16(exp(s - max) * (1/sum)) -- the
//    reference's rounding points, with the max and sum over all visible keys
//    -- and O += P V with P kept in registers (the score accumulator is the
//    next MMA's A fragment); out = bf16(O).
// Both contractions are mma.sync m16n8k16 (bf16 in, fp32 accumulate; bf16
// products are exact, so this is the reference's matmul up to summation
// order), fed by ldmatrix from padded shared-memory rows (272-byte stride:
// conflict-free).  K/V tiles stream through two buffers with cp.async; a warp
// stops at the last tile its rows can see (causal).  Query rows at or past
// the prompt length are written as zeros (they are padding).
#include "attention.cuh"

namespace sb {

namespace {

constexpr int kPfRows = 128;    // query rows per CTA
constexpr int kPfKeys = 64;     // keys per tile
constexpr int kPfStride = 136;  // shared-memory row stride in elements (272 bytes)
constexpr int kPfThreads = 256;
constexpr size_t kPfSmem = static_cast<size_t>(kPfRows + 4 * kPfKeys) * kPfStride * 2;  // Q + 2 x (K, V)

__device__ __forceinline__ uint32_t s32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t bf2(float lo, float hi) {  // two bf16 (round to nearest) in one word
  return static_cast<uint32_t>(f_to_bf16_bits(lo)) | (static_cast<uint32_t>(f_to_bf16_bits(hi)) << 16);
}

}  // namespace

struct PfArgs {
  const uint16_t* q;        // [B*T][n_q*128]
  const uint16_t* k_cache;  // [max_batch][n_kv][max_len][128]
  const uint16_t* v_cache;
  uint16_t* out;            // [B*T][n_q*128]
  const int32_t* prompt_len;
  int n_q, n_kv, max_len, T, qb_pos;
  float attn_mult;
};

__global__ void __launch_bounds__(kPfThreads, 2) k_attn_prefill(const __grid_constant__ PfArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint16_t* qs = reinterpret_cast<uint16_t*>(smem);  // [128][136]
  uint16_t* ksm = qs + kPfRows * kPfStride;           // [2][64][136]
  uint16_t* vsm = ksm + 2 * kPfKeys * kPfStride;      // [2][64][136]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int G = a.n_q / a.n_kv, QB = a.qb_pos;  // QB * G == 128
  const int qb = gridDim.x - 1 - blockIdx.x;    // the longest blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int q0 = qb * QB;
  const size_t tok0 = static_cast<size_t>(b) * a.T;
  const size_t rs = static_cast<size_t>(a.n_q) * 128;  // q / out row stride (elements)
  pdl_wait();
  pdl_launch();
  int plen = a.prompt_len ? a.prompt_len[b] : a.T;
  plen = plen > a.T ? a.T : plen;
  // row r of the CTA: position q0 + r / G, query head h * G + r % G
  auto out_row = [&](int r) { return a.out + (tok0 + q0 + r / G) * rs + (h * G + r % G) * 128; };
  if (q0 >= plen) {  // the whole block is padding
    for (int i = tid; i < kPfRows * 64; i += kPfThreads) {
      const int r = i >> 6;
      if (q0 + r / G < a.T) reinterpret_cast<uint32_t*>(out_row(r))[i & 63] = 0u;
    }
    return;
  }
  const int kmax = q0 + QB < plen ? q0 + QB : plen;  // keys any row of the block can see
  const int nkt = (kmax + kPfKeys - 1) / kPfKeys;
  const size_t head_row0 = (static_cast<size_t>(b) * a.n_kv + h) * a.max_len;
  auto load_tile = [&](uint16_t* dst, const uint16_t* cache, int kt) {
    for (int i = tid; i < kPfKeys * 16; i += kPfThreads) {
      const int r = i >> 4, ch = i & 15;
      int key = kt * kPfKeys + r;
      key = key < a.max_len ? key : a.max_len - 1;  // keys past the cache are masked; stay in bounds
      cp16(s32(dst + r * kPfStride + ch * 8), cache + (head_row0 + key) * 128 + ch * 8);
    }
  };
  for (int i = tid; i < kPfRows * 16; i += kPfThreads) {
    const int r = i >> 4, ch = i & 15;
    uint16_t* dst = qs + r * kPfStride + ch * 8;
    if (q0 + r / G < a.T)
      cp16(s32(dst), a.q + (tok0 + q0 + r / G) * rs + (h * G + r % G) * 128 + ch * 8);
    else
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
  load_tile(ksm, a.k_cache, 0);
  cp_commit();

  const int r0 = warp * 16;
  const int rowA = r0 + g, rowB = r0 + g + 8;  // this thread's two rows (fragment rows g, g + 8)
  const int posA = q0 + rowA / G, posB = q0 + rowB / G;
  int wlast = q0 + (r0 + 15) / G;  // the last key this warp's rows can see
  wlast = wlast < kmax - 1 ? wlast : kmax - 1;
  const int wkt = wlast / kPfKeys + 1;
  cp_wait_all();
  __syncthreads();
  // this warp's Q rows, read again from shared memory at every k-step (keeps
  // the registers of two CTAs per SM)
  const uint32_t qaddr = s32(qs + (r0 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kPfStride + 8 * (lane >> 4));

  float sacc[8][4];
  // rounded, masked scores of key tile kt (K in kbuf) -> sacc
  auto scores = [&](const uint16_t* kbuf, int kt) {
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) sacc[nt][j] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ks += 2) {
      uint32_t qa[4], qb2[4];
      ldsm4(qaddr + ks * 32, qa);
      ldsm4(qaddr + (ks + 1) * 32, qb2);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        uint32_t bfr[4];  // B fragments of k-steps ks and ks + 1 for keys 8 nt ..
        ldsm4(s32(kbuf + (nt * 8 + (lane & 7)) * kPfStride + ks * 16 + 8 * (lane >> 3)), bfr);
        mma_bf16(sacc[nt], qa, bfr[0], bfr[1]);
        mma_bf16(sacc[nt], qb2, bfr[2], bfr[3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int key = kt * kPfKeys + nt * 8 + 2 * c + (j & 1);
        const int pos = j < 2 ? posA : posB;
        const float s = bf(bf(sacc[nt][j]) * a.attn_mult);
        sacc[nt][j] = (key <= pos && key < plen) ? s : -INFINITY;
      }
  };

  // ---- pass 1: row max and exp-sum ----
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) load_tile(ksm + ((kt + 1) & 1) * kPfKeys * kPfStride, a.k_cache, kt + 1);
    cp_commit();
    if (kt < wkt) {
      scores(ksm + (kt & 1) * kPfKeys * kPfStride, kt);
      float tA = -INFINITY, tB = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        tA = fmaxf(tA, fmaxf(sacc[nt][0], sacc[nt][1]));
        tB = fmaxf(tB, fmaxf(sacc[nt][2], sacc[nt][3]));
      }
      tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, 1));
      tA = fmaxf(tA, __shfl_xor_sync(0xffffffffu, tA, 2));
      tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, 1));
      tB = fmaxf(tB, __shfl_xor_sync(0xffffffffu, tB, 2));
      // key 0 is visible to every row, so the max is finite from tile 0 on
      const float nA = fmaxf(mA, tA), nB = fmaxf(mB, tB);
      lA *= expf(mA - nA);
      lB *= expf(mB - nB);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        lA += expf(sacc[nt][0] - nA) + expf(sacc[nt][1] - nA);
        lB += expf(sacc[nt][2] - nB) + expf(sacc[nt][3] - nB);
      }
      mA = nA;
      mB = nB;
    }
    cp_wait_all();
    __syncthreads();
  }
  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  const float iA = 1.f / lA, iB = 1.f / lB;

  // ---- pass 2: P V ----
  load_tile(ksm, a.k_cache, 0);
  load_tile(vsm, a.v_cache, 0);
  cp_commit();
  cp_wait_all();
  __syncthreads();
  float oacc[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) oacc[nt][j] = 0.f;
  for (int kt = 0; kt < nkt; ++kt) {
    if (kt + 1 < nkt) {
      load_tile(ksm + ((kt + 1) & 1) * kPfKeys * kPfStride, a.k_cache, kt + 1);
      load_tile(vsm + ((kt + 1) & 1) * kPfKeys * kPfStride, a.v_cache, kt + 1);
    }
    cp_commit();
    if (kt < wkt) {
      scores(ksm + (kt & 1) * kPfKeys * kPfStride, kt);
      const uint16_t* vbuf = vsm + (kt & 1) * kPfKeys * kPfStride;
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {  // 16 keys per MMA k-step
        uint32_t pa[4];
        pa[0] = bf2(expf(sacc[2 * k2][0] - mA) * iA, expf(sacc[2 * k2][1] - mA) * iA);
        pa[1] = bf2(expf(sacc[2 * k2][2] - mB) * iB, expf(sacc[2 * k2][3] - mB) * iB);
        pa[2] = bf2(expf(sacc[2 * k2 + 1][0] - mA) * iA, expf(sacc[2 * k2 + 1][1] - mA) * iA);
        pa[3] = bf2(expf(sacc[2 * k2 + 1][2] - mB) * iB, expf(sacc[2 * k2 + 1][3] - mB) * iB);
#pragma unroll
        for (int n2 = 0; n2 < 8; ++n2) {  // 16 dims per ldmatrix
          uint32_t vb[4];
          ldsm4t(s32(vbuf + (k2 * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kPfStride + n2 * 16 + 8 * (lane >> 4)), vb);
          mma_bf16(oacc[2 * n2], pa, vb[0], vb[1]);
          mma_bf16(oacc[2 * n2 + 1], pa, vb[2], vb[3]);
        }
      }
    }
    cp_wait_all();
    __syncthreads();
  }
  // out = bf16(sum_j p_j v_j); rows at or past the prompt length are padding: zeros
  const bool okA = posA < a.T, okB = posB < a.T;
  const bool liveA = posA < plen, liveB = posB < plen;
  uint16_t* oA = out_row(rowA);
  uint16_t* oB = out_row(rowB);
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + 2 * c;
    if (okA) *reinterpret_cast<uint32_t*>(oA + d) = liveA ? bf2(oacc[nt][0], oacc[nt][1]) : 0u;
    if (okB) *reinterpret_cast<uint32_t*>(oB + d) = liveB ? bf2(oacc[nt][2], oacc[nt][3]) : 0u;
  }
}

bool attn_prefill_ok(int n_q, int n_kv) {
  if (n_kv < 1 || n_q % n_kv) return false;
  const int G = n_q / n_kv;
  return G >= 1 && kPfRows % G == 0 && kPfRows / G >= 8;
}

int attn_prefill_launch(const AttnParams& p, int batch, int T, cudaStream_t stream) {
  if (!attn_prefill_ok(p.n_q, p.n_kv) || T < 1 || T > p.max_len) return SB_ERR_CONFIG;
  PfArgs a;
  a.q = p.q;
  a.k_cache = p.k_cache;
  a.v_cache = p.v_cache;
  a.out = p.out;
  a.prompt_len = p.prompt_len;
  a.n_q = p.n_q;
  a.n_kv = p.n_kv;
  a.max_len = p.max_len;
  a.T = T;
  a.qb_pos = kPfRows / (p.n_q / p.n_kv);
  a.attn_mult = p.attn_mult;
  int dev = 0;
  cudaGetDevice(&dev);
  static unsigned configured = 0;
  if (!(configured & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kPfSmem));
    if (e != cudaSuccess) return e;
    configured |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((T + a.qb_pos - 1) / a.qb_pos, p.n_kv, batch);
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = kPfSmem;
  cfg.stream = stream;
  note_launch();
  return cudaLaunchKernelEx(&cfg, k_attn_prefill, a);
}

}  // namespace sb
