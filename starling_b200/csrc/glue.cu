// Standalone glue kernels (the reference's four Triton kernels and torch
// one-liners), exact dequantisation of the packed weight formats, and a
// row argmax.  The decode step itself uses the fused forms in gemv.cu; these
// exist as individually testable entry points with the reference's exact
// rounding points.
#include <algorithm>

#include "glue.cuh"

namespace sb {

// fused_rmsnorm (llm_kernels.py:93-139): y = w * bf16(x * rsqrt(mean(x^2) + eps))
__global__ void k_rmsnorm(const uint16_t* x, const uint16_t* w, uint16_t* y, int n, float eps) {
  const uint16_t* xr = x + static_cast<size_t>(blockIdx.x) * n;
  uint16_t* yr = y + static_cast<size_t>(blockIdx.x) * n;
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = u16_to_f(xr[i]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rstd = 1.f / sqrtf(red[0] / static_cast<float>(n) + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    yr[i] = f_to_bf16_bits(u16_to_f(w[i]) * bf(u16_to_f(xr[i]) * rstd));
}

// RMSNorm of whole rows for the decode step when it has more than 8 token
// rows (the GEMV prologue would otherwise recompute it in every CTA).  With
// ids != nullptr the row is first the embedding row times mult (rounded to
// bf16, llm_mega.py:514) and is also written to h_out (the residual stream).
__global__ void __launch_bounds__(256) k_norm_rows(const uint16_t* x, const int64_t* ids, const uint16_t* embed,
                                                   int embed_rows, float mult, const uint16_t* w, uint16_t* y,
                                                   uint16_t* h_out, int n, float eps) {
  pdl_wait();
  pdl_launch();
  const uint16_t* xr;
  if (ids) {
    int64_t id = ids[blockIdx.x];
    id = id < 0 ? 0 : (id >= embed_rows ? embed_rows - 1 : id);
    xr = embed + static_cast<size_t>(id) * n;
  } else {
    xr = x + static_cast<size_t>(blockIdx.x) * n;
  }
  uint16_t* yr = y + static_cast<size_t>(blockIdx.x) * n;
  __shared__ float red[8];
  float v[32];  // n <= 256 threads * 32
  int cnt = 0;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int k = threadIdx.x + i * 256;
    if (k < n) {
      float f = u16_to_f(xr[k]);
      if (ids) f = bf(f * mult);
      v[i] = f;
      ss += f * f;
      cnt = i + 1;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tsum = 0.f;
  for (int q = 0; q < 8; ++q) tsum += red[q];
  const float rstd = 1.f / sqrtf(tsum / static_cast<float>(n) + eps);
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int k = threadIdx.x + i * 256;
    if (i < cnt) {
      yr[k] = f_to_bf16_bits(u16_to_f(w[k]) * bf(v[i] * rstd));
      if (ids && h_out) h_out[static_cast<size_t>(blockIdx.x) * n + k] = f_to_bf16_bits(v[i]);
    }
  }
}

// fused_silu_mul (llm_kernels.py:241-285): bf16(silu(g)) * up
__global__ void k_silu_mul(const uint16_t* g, const uint16_t* u, uint16_t* o, int64_t count) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gv = u16_to_f(g[i]);
    o[i] = f_to_bf16_bits(bf(gv / (1.f + expf(-gv))) * u16_to_f(u[i]));
  }
}

// fused_residual_scale (llm_kernels.py:295-336): x + bf16(alpha * y)
__global__ void k_residual(const uint16_t* x, const uint16_t* y, uint16_t* z, int64_t count, float alpha) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    z[i] = f_to_bf16_bits(u16_to_f(x[i]) + bf(alpha * u16_to_f(y[i])));
}

// RoPE (llm_mega.py:538-543): q*cos + rotate_half(q)*sin, each product rounded
__global__ void k_rope(uint16_t* x, int rows, int heads, const int32_t* pos, const uint16_t* cs,
                       const uint16_t* sn) {
  const int r = blockIdx.x;
  const int j = threadIdx.x;  // 0..63
  if (r >= rows || j >= 64) return;
  uint16_t* xr = x + static_cast<size_t>(r) * 128;
  const int p = pos[r / heads];
  const float c = u16_to_f(cs[p * 64 + j]), s = u16_to_f(sn[p * 64 + j]);
  const float x1 = u16_to_f(xr[j]), x2 = u16_to_f(xr[j + 64]);
  xr[j] = f_to_bf16_bits(bf(x1 * c) - bf(x2 * s));
  xr[j + 64] = f_to_bf16_bits(bf(x2 * c) + bf(x1 * s));
}

// argmax over a bf16 row, first maximal index (torch semantics)
__global__ void k_argmax(const uint16_t* x, int n, int64_t* out) {
  const uint16_t* xr = x + static_cast<size_t>(blockIdx.x) * n;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = u16_to_f(xr[i]);
    if (am_better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (am_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w)
      if (am_better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
    out[blockIdx.x] = bi;
  }
}

// ---- exact dequantisation of a packed layer ------------------------------------
// One thread per (row tile, kgroup, lane): decodes its 16 bytes (8, 16 or 32
// elements) and writes them at their (row, k) positions.  The values are the
// oracle's: nvfp4 (code * e4m3) * g, fp8 e4m3 * s_row, int8 q * s_row.
__device__ __forceinline__ float h_lo(uint32_t h2) { return __half2float(__ushort_as_half(h2 & 0xffff)); }
__device__ __forceinline__ float h_hi(uint32_t h2) { return __half2float(__ushort_as_half(h2 >> 16)); }

template <typename OutT>
__device__ __forceinline__ void store_out(OutT* o, size_t i, float v);
template <>
__device__ __forceinline__ void store_out<float>(float* o, size_t i, float v) { o[i] = v; }
template <>
__device__ __forceinline__ void store_out<uint16_t>(uint16_t* o, size_t i, float v) { o[i] = f_to_bf16_bits(v); }

template <typename OutT>
__global__ void k_dequant(SbLinear lin, OutT* out) {
  const int kge = lin.fmt == SB_FMT_NVFP4 ? 64 : (lin.fmt == SB_FMT_BF16 ? 16 : 32);
  const int kg_total = lin.k / kge;
  const size_t total = static_cast<size_t>(lin.n_pad / 16) * kg_total * 32;
  const size_t gid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (gid >= total) return;
  const int lane = static_cast<int>(gid & 31);
  const size_t tk = gid >> 5;
  const int kg = static_cast<int>(tk % kg_total);
  const int tile = static_cast<int>(tk / kg_total);
  const int g = lane >> 2, c = lane & 3;
  const uint4 a = reinterpret_cast<const uint4*>(lin.w)[gid];
  const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
  // fragment element e -> (row offset, k offset) within a 16x16 k-step
  const int rofs[8] = {g, g, g + 8, g + 8, g, g, g + 8, g + 8};
  const int kofs[8] = {2 * c, 2 * c + 1, 2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9, 2 * c + 8, 2 * c + 9};
  const int ksteps = kge / 16;
  for (int ks = 0; ks < ksteps; ++ks) {
    float v[8];
    if (lin.fmt == SB_FMT_NVFP4) {
      const uint2 s = reinterpret_cast<const uint2*>(lin.scale)[(static_cast<size_t>(tile) * kg_total + kg) * 8 + g];
      const uint32_t sp = ((ks < 2) ? s.x : s.y) >> ((ks & 1) * 16);
      const uint32_t sh = e4m3x2_to_h2(sp);
      const float s_lo = h_lo(sh), s_hi = h_hi(sh);
      for (int q = 0; q < 4; ++q) {
        const uint32_t h = e2m1x2_to_h2(wv[ks] >> (8 * q));
        const float sc = (q & 1) ? s_hi : s_lo;  // bytes 0,2 -> row g; 1,3 -> row g+8
        v[2 * q] = (h_lo(h) * sc) * lin.global_scale;
        v[2 * q + 1] = (h_hi(h) * sc) * lin.global_scale;
      }
    } else if (lin.fmt == SB_FMT_FP8 || lin.fmt == SB_FMT_INT8) {
      const uint32_t w0 = wv[2 * ks], w1 = wv[2 * ks + 1];
      uint32_t h[4];
      if (lin.fmt == SB_FMT_FP8) {
        h[0] = e4m3x2_to_h2(w0);
        h[1] = e4m3x2_to_h2(w0 >> 16);
        h[2] = e4m3x2_to_h2(w1);
        h[3] = e4m3x2_to_h2(w1 >> 16);
      } else {
        i8x4_to_h2x2(w0, h[0], h[1]);
        i8x4_to_h2x2(w1, h[2], h[3]);
      }
      const float* rs = reinterpret_cast<const float*>(lin.scale);
      for (int q = 0; q < 4; ++q) {
        const int row = tile * 16 + rofs[2 * q];
        v[2 * q] = h_lo(h[q]) * rs[row];
        v[2 * q + 1] = h_hi(h[q]) * rs[row];
      }
    } else {
      for (int q = 0; q < 4; ++q) {
        v[2 * q] = __uint_as_float(wv[q] << 16);
        v[2 * q + 1] = __uint_as_float(wv[q] & 0xffff0000u);
      }
    }
    for (int e = 0; e < 8; ++e) {
      const int row = tile * 16 + rofs[e];
      if (row >= lin.n) continue;
      const size_t k = static_cast<size_t>(kg) * kge + ks * 16 + kofs[e];
      store_out<OutT>(out, static_cast<size_t>(row) * lin.k + k, v[e]);
    }
  }
}

template __global__ void k_dequant<float>(SbLinear, float*);
template __global__ void k_dequant<uint16_t>(SbLinear, uint16_t*);

int dequant_launch(const SbLinear& lin, void* out, bool f32, cudaStream_t s) {
  const int kge = lin.fmt == SB_FMT_NVFP4 ? 64 : (lin.fmt == SB_FMT_BF16 ? 16 : 32);
  const size_t total = static_cast<size_t>(lin.n_pad / 16) * (lin.k / kge) * 32;
  const int bs = 256;
  const unsigned grid = static_cast<unsigned>((total + bs - 1) / bs);
  note_launch();
  if (f32)
    k_dequant<float><<<grid, bs, 0, s>>>(lin, static_cast<float*>(out));
  else
    k_dequant<uint16_t><<<grid, bs, 0, s>>>(lin, static_cast<uint16_t*>(out));
  return cudaGetLastError();
}

int norm_rows_launch(const uint16_t* x, const int64_t* ids, const uint16_t* embed, int embed_rows, float mult,
                     const uint16_t* w, uint16_t* y, uint16_t* h_out, int rows, int n, float eps, bool pdl,
                     cudaStream_t s) {
  if (n > 256 * 32) return SB_ERR_CONFIG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  note_launch();
  return cudaLaunchKernelEx(&cfg, k_norm_rows, x, ids, embed, embed_rows, mult, w, y, h_out, n, eps);
}

int rmsnorm_launch(const uint16_t* x, const uint16_t* w, uint16_t* y, int rows, int n, float eps, cudaStream_t s) {
  note_launch();
  k_rmsnorm<<<rows, 256, 0, s>>>(x, w, y, n, eps);
  return cudaGetLastError();
}
int silu_mul_launch(const uint16_t* g, const uint16_t* u, uint16_t* o, int64_t count, cudaStream_t s) {
  const int grid = static_cast<int>(std::min<int64_t>((count + 255) / 256, 148 * 16));
  note_launch();
  k_silu_mul<<<grid > 0 ? grid : 1, 256, 0, s>>>(g, u, o, count);
  return cudaGetLastError();
}
int residual_launch(const uint16_t* x, const uint16_t* y, uint16_t* z, int64_t count, float alpha, cudaStream_t s) {
  const int grid = static_cast<int>(std::min<int64_t>((count + 255) / 256, 148 * 16));
  note_launch();
  k_residual<<<grid > 0 ? grid : 1, 256, 0, s>>>(x, y, z, count, alpha);
  return cudaGetLastError();
}
int rope_launch(uint16_t* x, int rows, int heads, const int32_t* pos, const uint16_t* cs, const uint16_t* sn,
                cudaStream_t s) {
  note_launch();
  k_rope<<<rows, 64, 0, s>>>(x, rows, heads, pos, cs, sn);
  return cudaGetLastError();
}
int argmax_launch(const uint16_t* x, int rows, int n, int64_t* out, cudaStream_t s) {
  note_launch();
  k_argmax<<<rows, 1024, 0, s>>>(x, n, out);
  return cudaGetLastError();
}

}  // namespace sb

namespace sb {

// Control block of a prefill: cache slot of token 0, padded prompt length, the rest zero.
__global__ void k_set_ctrl(int32_t* ctrl, int slot, int padlen) {
  const int i = threadIdx.x;
  if (i < SB_CTRL_WORDS) ctrl[i] = i == SB_CTRL_SLOT ? slot : (i == SB_CTRL_PADLEN ? padlen : 0);
}

int set_ctrl_launch(int32_t* ctrl, int slot, int padlen, cudaStream_t s) {
  note_launch();
  k_set_ctrl<<<1, 32, 0, s>>>(ctrl, slot, padlen);
  return cudaGetLastError();
}

}  // namespace sb
