// Decode / verify attention over the static KV cache, sm_100a.
//
// Replaces the reference's per-layer attention block
// (src/starling/granite/llm_mega.py:549-556 and the HF eager path
// transformers modeling_granite.py:89-112): repeat_kv copies of K/V, a
// scores matmul over all max_cache_len slots, an additive -max mask, an fp32
// softmax cast to bf16 and a probs @ V matmul.  Here:
//  * no repeat_kv: one cluster serves one (stream, KV head) and all of its
//    query heads (and, for verify, all query tokens) at once;
//  * only keys that can be valid are read: [0, slot + m) with right-padding
//    holes [prompt_len, pad_len) skipped, which is exactly the set the
//    reference's mask leaves at 0 (masked slots contribute exp(-inf) = 0);
//  * the `split` CTAs of a cluster each take a slice of the keys; the
//    softmax max and sum and the P.V partials are combined across the
//    cluster through distributed shared memory in a fixed order;
//  * rounding points follow the reference: score = bf16(bf16(q.k) * scale),
//    p = bf16(exp(s - max) * (1/sum)) in fp32, out = bf16(sum_j p_j v_j).
#include <cooperative_groups.h>

#include "attention.cuh"

namespace cg = cooperative_groups;

namespace sb {

__global__ void __launch_bounds__(256) k_attn(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  cg::cluster_group cl = cg::this_cluster();
  const int rank = static_cast<int>(cl.block_rank());
  const int split = p.split;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.n_q / p.n_kv;
  const int R = G * p.m_per;

  const int slot = p.ctrl[SB_CTRL_SLOT];
  const int pad_len = p.ctrl[SB_CTRL_PADLEN];
  const int plen = p.prompt_len ? p.prompt_len[b] : 0x7fffffff;
  int kv_len = slot + p.m_per;
  kv_len = kv_len > p.max_len ? p.max_len : kv_len;
  const int chunk = (kv_len + split - 1) / split;
  const int lo = rank * chunk;
  const int hi = min(kv_len, lo + chunk);
  const int nk = hi > lo ? hi - lo : 0;

  const size_t head_base = (static_cast<size_t>(b) * p.n_kv + kvh) * p.max_len;
  const uint16_t* kc = p.k_cache + head_base * 128;
  const uint16_t* vc = p.v_cache + head_base * 128;
  if (tid == 0 && nk > 0) {
    prefetch_l2(kc + static_cast<size_t>(lo) * 128, static_cast<uint32_t>(nk) * 256u);
    prefetch_l2(vc + static_cast<size_t>(lo) * 128, static_cast<uint32_t>(nk) * 256u);
  }
  pdl_wait();
  pdl_launch();

  float* qs = reinterpret_cast<float*>(smem);        // [R][128]
  float* sc = qs + R * 128;                          // [R][chunk_cap]
  float* part = sc + R * p.chunk_cap;                // [16][4][128]
  float* outp = part + 16 * 4 * 128;                 // [R][128]
  float* smax = outp + R * 128;                      // [R]
  float* ssum = smax + 128;                          // [R]

  // q rows of this KV group: row r = (token mi, head gi)
  for (int i = tid; i < R * 128; i += blockDim.x) {
    const int r = i >> 7, d = i & 127;
    const int mi = r / G, gi = r % G;
    const size_t t = static_cast<size_t>(b) * p.m_per + mi;
    qs[i] = u16_to_f(p.q[t * p.n_q * 128 + (kvh * G + gi) * 128 + d]);
  }
  __syncthreads();

  // ---- scores: a half-warp per key, 8 dims per lane --------------------------------
  const int hw = tid >> 4, l16 = tid & 15;
  // Both half-warps of a warp run the same trip count (the shuffles below
  // use the full mask); the odd key of a pair past the end is predicated off.
  for (int jb = hw & ~1; jb < nk; jb += 16) {
    const int jj = jb + (hw & 1);
    const bool live = jj < nk;
    const int j = lo + (live ? jj : 0);
    float kf[8];
    {
      uint4 v = make_uint4(0, 0, 0, 0);
      if (live) v = *reinterpret_cast<const uint4*>(kc + static_cast<size_t>(j) * 128 + l16 * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kf[2 * i] = __uint_as_float(w[i] << 16);
        kf[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
    const bool hole = j >= plen && j < pad_len;
    for (int r = 0; r < R; ++r) {
      const float* qr = qs + r * 128 + l16 * 8;
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(qr[i], kf[i], d);
      d += __shfl_xor_sync(0xffffffffu, d, 8);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      if (l16 == 0 && live) {
        const int mi = r / G;
        const bool valid = !hole && j <= slot + mi;
        sc[r * p.chunk_cap + jj] = valid ? bf(bf(d) * p.attn_mult) : -INFINITY;
      }
    }
  }
  __syncthreads();

  // ---- softmax statistics across the cluster ------------------------------------------
  for (int r = warp; r < R; r += 8) {
    float m = -INFINITY;
    for (int jj = lane; jj < nk; jj += 32) m = fmaxf(m, sc[r * p.chunk_cap + jj]);
    m = warp_max(m);
    if (lane == 0) smax[r] = m;
  }
  cl.sync();
  for (int r = warp; r < R; r += 8) {
    float gm = -INFINITY;
    for (int q = 0; q < split; ++q) gm = fmaxf(gm, cl.map_shared_rank(smax, q)[r]);
    float s = 0.f;
    for (int jj = lane; jj < nk; jj += 32) {
      float* e = sc + r * p.chunk_cap + jj;
      const float ev = gm == -INFINITY ? 0.f : expf(*e - gm);
      *e = ev;
      s += ev;
    }
    s = warp_sum(s);
    if (lane == 0) ssum[r] = s;
  }
  cl.sync();
  for (int r = warp; r < R; r += 8) {
    float gs = 0.f;
    for (int q = 0; q < split; ++q) gs += cl.map_shared_rank(ssum, q)[r];
    const float inv = 1.f / gs;
    for (int jj = lane; jj < nk; jj += 32) {
      float* e = sc + r * p.chunk_cap + jj;
      *e = bf(*e * inv);  // softmax(..., dtype=float32).to(bf16)
    }
  }
  __syncthreads();

  // ---- P.V partial: thread = (key group kg, 8 dims dc), rows in blocks of 4 ---------
  const int dc = tid & 15, kgp = tid >> 4;
  for (int r0 = 0; r0 < R; r0 += 4) {
    const int nr = min(4, R - r0);
    float acc[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[a][i] = 0.f;
    for (int jj = kgp; jj < nk; jj += 16) {
      const uint4 v = *reinterpret_cast<const uint4*>(vc + static_cast<size_t>(lo + jj) * 128 + dc * 8);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      float vf[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        vf[2 * i] = __uint_as_float(w[i] << 16);
        vf[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        if (a < nr) {
          const float pr = sc[(r0 + a) * p.chunk_cap + jj];
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[a][i] = fmaf(pr, vf[i], acc[a][i]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int i = 0; i < 8; ++i) part[(kgp * 4 + a) * 128 + dc * 8 + i] = acc[a][i];
    __syncthreads();
    for (int i = tid; i < nr * 128; i += blockDim.x) {
      const int a = i >> 7, d = i & 127;
      float s = 0.f;
      for (int q = 0; q < 16; ++q) s += part[(q * 4 + a) * 128 + d];
      outp[(r0 + a) * 128 + d] = s;
    }
    __syncthreads();
  }

  // ---- combine the cluster's partial outputs, round, store -----------------------------
  cl.sync();
  if (rank == 0) {
    for (int i = tid; i < R * 128; i += blockDim.x) {
      float s = 0.f;
      for (int q = 0; q < split; ++q) s += cl.map_shared_rank(outp, q)[i];
      const int r = i >> 7, d = i & 127;
      const int mi = r / G, gi = r % G;
      const size_t t = static_cast<size_t>(b) * p.m_per + mi;
      p.out[t * p.n_q * 128 + (kvh * G + gi) * 128 + d] = f_to_bf16_bits(s);
    }
  }
  cl.sync();
}

size_t attn_smem_bytes(int R, int chunk_cap) {
  return (static_cast<size_t>(R) * 128 * 2 + static_cast<size_t>(R) * chunk_cap + 16 * 4 * 128 + 128 * 2) * 4 + 16;
}

int attn_launch(const AttnParams& p, int batch, bool pdl, cudaStream_t stream) {
  const int R = (p.n_q / p.n_kv) * p.m_per;
  if (R > 128 || R < 1 || p.split < 1 || p.split > 8) return SB_ERR_CONFIG;
  const size_t smem = attn_smem_bytes(R, p.chunk_cap);
  if (smem > 200 * 1024) return SB_ERR_CONFIG;
  int dev = 0;
  cudaGetDevice(&dev);
  static unsigned configured = 0;
  if (!(configured & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    configured |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.split, p.n_kv, batch);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = p.split;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  int na = 1;
  if (pdl) {
    attrs[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[1].val.programmaticStreamSerializationAllowed = 1;
    na = 2;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, k_attn, p);
}

}  // namespace sb
