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

}  // namespace sb
