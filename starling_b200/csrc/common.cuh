// Shared device helpers for the starling_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/starling_b200.h"

namespace sb {

typedef __nv_bfloat16 bf16;

// Kernels launched by this library (host-side counter, reported by sb_launch_count).
void note_launch();
// Record the message sb_last_error() returns; returns `code`.
int set_error(int code, const char* fmt, ...);

// ---- rounding helpers -----------------------------------------------------
// Every reference op rounds its result to bf16; these make the rounding
// points explicit.
__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float ld_bf(const uint16_t* p) {
  return __bfloat162float(*reinterpret_cast<const bf16*>(p));
}
__device__ __forceinline__ float u16_to_f(uint16_t u) {
  return __uint_as_float(static_cast<uint32_t>(u) << 16);
}
__device__ __forceinline__ uint16_t f_to_bf16_bits(float x) {
  bf16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}

// ---- loads ------------------------------------------------------------------
// Streaming weight loads: read-only path, do not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ldg_stream2(const uint2* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

// Bulk prefetch of [p, p+bytes) into L2 (p 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- programmatic dependent launch -------------------------------------------
// wait: block until the preceding kernel in the stream has completed and its
// writes are visible (no-op when launched without the PDL attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// allow the next kernel in the stream to be scheduled (it still waits for
// this one to complete before touching our outputs).
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// ---- tensor-core fragments (mma.sync m16n8k16, fp32 accumulate) ----------------
__device__ __forceinline__ void mma_f16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_bf16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- weight decoding into f16x2 A-fragment registers -------------------------
__device__ __forceinline__ uint32_t e2m1x2_to_h2(uint32_t byte) {
  __half2_raw r = __nv_cvt_fp4x2_to_halfraw2(static_cast<__nv_fp4x2_storage_t>(byte & 0xFF), __NV_E2M1);
  return static_cast<uint32_t>(r.x) | (static_cast<uint32_t>(r.y) << 16);
}
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t two) {
  __half2_raw r = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xFFFF), __NV_E4M3);
  return static_cast<uint32_t>(r.x) | (static_cast<uint32_t>(r.y) << 16);
}
// four signed int8 (bytes b0..b3 of w) -> two f16x2 {b0,b1}, {b2,b3}; exact.
__device__ __forceinline__ void i8x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t x = w ^ 0x80808080u;  // b + 128 as unsigned bytes
  lo = __byte_perm(x, 0x64646464u, 0x7170);
  hi = __byte_perm(x, 0x64646464u, 0x7372);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  __half2 l = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
  __half2 h = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
  lo = *reinterpret_cast<uint32_t*>(&l);
  hi = *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// ---- 8 x bf16 <-> fp32 ---------------------------------------------------------
__device__ __forceinline__ void unpack8(const uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = static_cast<uint32_t>(f_to_bf16_bits(f[2 * i])) | (static_cast<uint32_t>(f_to_bf16_bits(f[2 * i + 1])) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ---- reductions --------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// argmax ordering: larger value wins, ties go to the lower index (torch).
__device__ __forceinline__ bool am_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

}  // namespace sb
