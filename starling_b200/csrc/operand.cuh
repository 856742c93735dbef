// The activation operand of the tensor-core GEMM (gemm_tc.cu): its byte
// layout and the fp8 two-term split, shared by the operand preparation and
// by kernels that write the operand of the next GEMM directly (attention.cu).
#pragma once
#include "common.cuh"

namespace sb {

// Byte offset of 16-byte chunk c (along K bytes) of operand row n in one token
// tile [kb][np/8][8 chunks][8 rows][16 B] (kb_bytes = np * 128): every 128-byte
// K block is contiguous in the no-swizzle K-major canonical layout of
// tcgen05.mma.
__host__ __device__ __forceinline__ size_t tc_operand_offset(size_t kb_bytes, int n, int c) {
  return static_cast<size_t>(c >> 3) * kb_bytes + static_cast<size_t>(n >> 3) * 1024 + (c & 7) * 128 + (n & 7) * 16;
}

// power-of-two scale of an fp8 operand row (or row slice) with largest
// magnitude am: max |x| 2^shift in [128, 256)
__device__ __forceinline__ int tc_fp8_shift(float am) {
  int e2 = 0;
  if (am > 0.f) frexpf(am, &e2);
  return 8 - e2;
}

// 16 activation values -> the two e4m3 terms of the fp8 operand, x 2^shift =
// t0 + t1 / 16 with t0 = e4m3(x 2^shift), t1 = e4m3(16 (x 2^shift - t0)), both
// round-to-nearest saturating, bytes in element order.  The power-of-two
// scaling and both subtractions are exact; the conversions go two at a time.
__device__ __forceinline__ void e4m3_split16(const float* f, int shift, uint4& w0, uint4& w1) {
  const bool fast = shift >= -126 && shift <= 126;  // 2^shift is a normal float
  const float s2 = fast ? __int_as_float((shift + 127) << 23) : 0.f;
  uint32_t a[4], b[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float v[4], r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = fast ? f[4 * i + e] * s2 : ldexpf(f[4 * i + e], shift);
    const uint32_t p0 = __nv_cvt_float2_to_fp8x2(make_float2(v[0], v[1]), __NV_SATFINITE, __NV_E4M3);
    const uint32_t p1 = __nv_cvt_float2_to_fp8x2(make_float2(v[2], v[3]), __NV_SATFINITE, __NV_E4M3);
    const float2 d0 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(p0), __NV_E4M3)));
    const float2 d1 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(p1), __NV_E4M3)));
    r[0] = (v[0] - d0.x) * 16.f;
    r[1] = (v[1] - d0.y) * 16.f;
    r[2] = (v[2] - d1.x) * 16.f;
    r[3] = (v[3] - d1.y) * 16.f;
    const uint32_t p2 = __nv_cvt_float2_to_fp8x2(make_float2(r[0], r[1]), __NV_SATFINITE, __NV_E4M3);
    const uint32_t p3 = __nv_cvt_float2_to_fp8x2(make_float2(r[2], r[3]), __NV_SATFINITE, __NV_E4M3);
    a[i] = (p0 & 0xFFFFu) | (p1 << 16);
    b[i] = (p2 & 0xFFFFu) | (p3 << 16);
  }
  w0 = make_uint4(a[0], a[1], a[2], a[3]);
  w1 = make_uint4(b[0], b[1], b[2], b[3]);
}

// ---- block-scaled fp8 operand ---------------------------------------------------
// The operand a producing GEMM epilogue writes for the next decode projection
// (tcgen05.mma kind::mxf8f6f4 with UE8M0 scales on B): per 128-element K
// block, np rows x 128 B of e4m3 in the layout above, then 512 B of scales,
// one per (row, 32-element block): byte (n % 32) * 16 + (n / 32) * 4 + j for
// row n < 128 and block j of the K block -- the layout tcgen05.cp
// .32x128b.warpx4 copies into four TMEM columns (row n's four scales in
// column n / 32 of lane n % 32).  Token m's terms are rows m and mp + m,
// x 2^s = t0 + t1 / 16 with s per (token, 32-element block).
__host__ __device__ __forceinline__ size_t tc_bs_block_bytes(int np) { return static_cast<size_t>(np) * 128 + 512; }
__host__ __device__ __forceinline__ size_t tc_bs_byte(int np, int n, int k) {
  return static_cast<size_t>(k >> 7) * tc_bs_block_bytes(np) + static_cast<size_t>(n >> 3) * 1024 + ((k >> 4) & 7) * 128 +
         (n & 7) * 16 + (k & 15);
}
__host__ __device__ __forceinline__ size_t tc_bs_scale_byte(int np, int n, int k) {
  return static_cast<size_t>(k >> 7) * tc_bs_block_bytes(np) + static_cast<size_t>(np) * 128 + (n & 31) * 16 +
         (n >> 5) * 4 + ((k >> 5) & 3);
}
// the block scale's exponent: max |x| 2^shift in [128, 256), kept where 2^shift
// and the UE8M0 code 127 - shift stay normal
__device__ __forceinline__ int tc_bs_shift(float am) {
  const int s = tc_fp8_shift(am);
  return s < -126 ? -126 : (s > 126 ? 126 : s);
}
// one value's two e4m3 terms: x 2^shift = t0 + t1 / 16 (as e4m3_split16)
__device__ __forceinline__ void e4m3_split1(float x, int shift, uint32_t& t0, uint32_t& t1) {
  const float v = x * __int_as_float((shift + 127) << 23);
  const uint32_t p0 = __nv_cvt_float2_to_fp8x2(make_float2(v, 0.f), __NV_SATFINITE, __NV_E4M3);
  const float2 d0 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(p0), __NV_E4M3)));
  const uint32_t p1 = __nv_cvt_float2_to_fp8x2(make_float2((v - d0.x) * 16.f, 0.f), __NV_SATFINITE, __NV_E4M3);
  t0 = p0 & 0xFFu;
  t1 = p1 & 0xFFu;
}
// 8 values -> their two e4m3 terms (as e4m3_split16), bytes in element order
__device__ __forceinline__ void e4m3_split8(const float* f, int shift, uint2& w0, uint2& w1) {
  const float s2 = __int_as_float((shift + 127) << 23);  // shift in [-126, 126]: a normal float
  uint32_t a[2], b[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    float v[4], r[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = f[4 * i + e] * s2;
    const uint32_t p0 = __nv_cvt_float2_to_fp8x2(make_float2(v[0], v[1]), __NV_SATFINITE, __NV_E4M3);
    const uint32_t p1 = __nv_cvt_float2_to_fp8x2(make_float2(v[2], v[3]), __NV_SATFINITE, __NV_E4M3);
    const float2 d0 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(p0), __NV_E4M3)));
    const float2 d1 = __half22float2(__half2(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(p1), __NV_E4M3)));
    r[0] = (v[0] - d0.x) * 16.f;
    r[1] = (v[1] - d0.y) * 16.f;
    r[2] = (v[2] - d1.x) * 16.f;
    r[3] = (v[3] - d1.y) * 16.f;
    const uint32_t p2 = __nv_cvt_float2_to_fp8x2(make_float2(r[0], r[1]), __NV_SATFINITE, __NV_E4M3);
    const uint32_t p3 = __nv_cvt_float2_to_fp8x2(make_float2(r[2], r[3]), __NV_SATFINITE, __NV_E4M3);
    a[i] = (p0 & 0xFFFFu) | (p1 << 16);
    b[i] = (p2 & 0xFFFFu) | (p3 << 16);
  }
  w0 = make_uint2(a[0], a[1]);
  w1 = make_uint2(b[0], b[1]);
}

// Token rows m0 + [0, M) x elements [k0, k0 + nk) of the block-scaled operand
// (k0, nk multiples of 32), from shared memory sv[m * nk + j], each value
// first multiplied by g[k0 + j] (bf16; null: by 1).  ssq (non-null) receives,
// per (token, 32-element block), the sum of squares of the values before that
// multiply: ssq[(m0 + m) * ssq_ld + (k0 + j) / 32].  Threads tid < nthr (a
// multiple of 32: a warp or more) take part with uniform arguments; each
// takes 8 consecutive elements, four consecutive lanes one 32-element block.
__device__ __forceinline__ void tc_bs_write_tile(uint8_t* op, int np, int mp, int m0, int k0, int nk, const float* sv,
                                                 int M, const uint16_t* g, float* ssq, int ssq_ld, int tid, int nthr) {
  const int ng = nk >> 3;  // 8-element groups per token row (a multiple of 4)
  const int U = M * ng;
  for (int base = 0; base < U; base += nthr) {
    const int u = base + tid;
    const bool on = u < U;
    const int m = on ? u / ng : 0, j8 = on ? (u - m * ng) * 8 : 0;
    float x[8];
    if (on) {
      const float4 a = *reinterpret_cast<const float4*>(sv + m * nk + j8);
      const float4 b = *reinterpret_cast<const float4*>(sv + m * nk + j8 + 4);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
      x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = 0.f;
    }
    float sq = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) sq += x[e] * x[e];
    if (g && on) {
      float w[8];
      unpack8(*reinterpret_cast<const uint4*>(g + k0 + j8), w);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] *= w[e];
    }
    float am = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(x[e]));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    sq += __shfl_xor_sync(0xffffffffu, sq, 1);
    sq += __shfl_xor_sync(0xffffffffu, sq, 2);
    if (on) {
      const int sh = tc_bs_shift(am);
      uint2 w0, w1;
      e4m3_split8(x, sh, w0, w1);
      const int k = k0 + j8;
      const int n = m0 + m;
      *reinterpret_cast<uint2*>(op + tc_bs_byte(np, n, k)) = w0;
      *reinterpret_cast<uint2*>(op + tc_bs_byte(np, mp + n, k)) = w1;
      if ((j8 & 31) == 0) {
        op[tc_bs_scale_byte(np, n, k)] = static_cast<uint8_t>(127 - sh);
        op[tc_bs_scale_byte(np, mp + n, k)] = static_cast<uint8_t>(127 - sh);
        if (ssq) ssq[static_cast<size_t>(n) * ssq_ld + (k >> 5)] = sq;
      }
    }
  }
}

}  // namespace sb
