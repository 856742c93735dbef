// Persistent decode GEMV for up to 8 token rows, sm_100a.
//
// Same operation and epilogues as k_gemv (gemv.cu), organised for the B=1
// decode regime where every kernel is small and latency decides:
//  * one wave: at most one CTA per SM, each owning a contiguous range of
//    16-row tiles of the (packed) weight;
//  * the CTA's weight tiles are streamed by bulk copies
//    (cp.async.bulk ... mbarrier::complete_tx) into a ring of shared-memory
//    slots; the first ring-full is issued BEFORE griddepcontrol.wait, so it
//    overlaps the previous kernel;
//  * the activation rows are read once per CTA, straight into registers in
//    mma B-fragment order: warp w owns K slice w for every tile, so its
//    fragments are reused across all of the CTA's tiles (no shared-memory
//    staging).  RMSNorm statistics are combined across warps in a fixed
//    order; each warp scales its slice by its own power of two (exact
//    bf16 -> f16) and undoes it on its partial sums;
//  * weight fragments are decoded from shared memory (e2m1 / e4m3 / int8 ->
//    f16 with PTX cvt, NVFP4 block scale applied as an exact f16 product) into
//    mma.m16n8k16 with fp32 accumulation; per-tile partials of all warps are
//    reduced through shared memory in a fixed order, a batch of tiles at a
//    time, while the other half of the ring is in flight.
// Every wait on the ring is bounded; on expiry the kernel records an error
// in ctrl[SB_CTRL_ERR] and carries on (results are then invalid) instead of
// hanging.
#include "gemv.cuh"
#include "gemv_epi.cuh"

namespace sb {

namespace {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// e2m1x2 bytes of one 32-bit word -> four f16x2 registers (PTX cvt, sm_100a)
__device__ __forceinline__ void e2m1x8_to_h2x4(uint32_t w, uint32_t& a0, uint32_t& a1, uint32_t& a2, uint32_t& a3) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}\n"
      : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
      : "r"(w));
}
__device__ __forceinline__ void e4m3x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n .reg .b16 l, h;\n mov.b32 {l, h}, %2;\n cvt.rn.f16x2.e4m3x2 %0, l;\n cvt.rn.f16x2.e4m3x2 %1, h;\n}\n"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

constexpr long kSpinLimit = 1L << 26;  // bounded waits (~seconds), then flag an error

__device__ __forceinline__ void ring_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  long it = 0;
  while (!mbar_try_wait(bar, parity)) {
    if (++it > kSpinLimit) {
      if (err) atomicExch(err, 1);
      return;
    }
  }
}

}  // namespace

template <int FMT, int KSW>
__global__ void __launch_bounds__(512, 2) k_gemv_dec(const __grid_constant__ GemvParams p, int slots, int batch) {
  constexpr int KGE = KG<FMT>::E;
  constexpr int KS = KGE / 16;
  constexpr int KPW = KSW / KS;  // kgroups per warp
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, W = blockDim.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int M = p.m;  // 1..8
  const int nct = gridDim.x;
  const int base = p.n_tiles / nct, extra = p.n_tiles % nct;
  const int ntile = base + (static_cast<int>(blockIdx.x) < extra ? 1 : 0);
  const int t0 = static_cast<int>(blockIdx.x) * base + min(static_cast<int>(blockIdx.x), extra);

  const uint32_t wbytes = static_cast<uint32_t>(p.kg_total) * 512u;
  const uint32_t sbytes = FMT == SB_FMT_NVFP4 ? static_cast<uint32_t>(p.kg_total) * 64u : 0u;
  const DecLayout L = dec_layout(wbytes + sbytes, slots, batch, W, M, KSW * 16);
  const uint32_t slot_bytes = static_cast<uint32_t>(L.slot_bytes);
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  float* red = reinterpret_cast<float*>(smem + L.red);     // [batch][W][16][M]
  float* tot = reinterpret_cast<float*>(smem + L.tot);     // [batch*16][M]
  float* s_ss = reinterpret_cast<float*>(smem + L.ss);     // [16 warps][8 rows]
  int* s_best = reinterpret_cast<int*>(smem + L.best);     // [8]
  float* s_bval = reinterpret_cast<float*>(smem + L.bval); // [8]
  int* s_flag = reinterpret_cast<int*>(smem + L.flag);
  int32_t* err = p.ctrl ? p.ctrl + SB_CTRL_ERR : nullptr;

  auto issue_tile = [&](int j) {  // tile j of this CTA -> slot j % slots
    uint8_t* dst = ring + static_cast<size_t>(j % slots) * slot_bytes;
    uint64_t* bar = bars + (j % slots);
    const size_t t = static_cast<size_t>(t0 + j);
    mbar_expect_tx(bar, wbytes + sbytes);
    const uint8_t* src = p.w + t * wbytes;
    for (uint32_t o = 0; o < wbytes; o += 32768u) bulk_g2s(dst + o, src + o, min(32768u, wbytes - o), bar);
    if (sbytes) bulk_g2s(dst + wbytes, p.scale + t * sbytes, sbytes, bar);
  };

  // ---- 1. start streaming this CTA's weights, then wait for the producer ----
  if (tid == 0) {
    for (int s = 0; s < slots; ++s) mbar_init(bars + s, 1);
    mbar_fence_init();
    for (int j = 0; j < min(slots, ntile); ++j) issue_tile(j);
  }
  __syncthreads();
  pdl_wait();
  pdl_launch();

  // ---- 2. activation rows -> this warp's K slice, f16 (or bf16), in shared memory
  // Warp w owns K slice w for every tile of the CTA.  Compact, rolled loops:
  // this code runs once per launch, so instruction fetch (not ALU) decides.
  const int Kw = KSW * 16;  // K elements per warp
  const int k0 = warp * Kw;
  const int xstride = Kw + 8;
  uint16_t* xw = reinterpret_cast<uint16_t*>(smem + L.xs) + static_cast<size_t>(warp) * M * xstride;
  int* s_shift = reinterpret_cast<int*>(smem + L.shift);  // [16 warps][8 rows]
  const bool embed = p.pro == PRO_EMBED;
  auto row_src = [&](int m) -> const uint16_t* {
    if (embed) {
      int64_t id = p.ids[m];
      id = id < 0 ? 0 : (id >= p.embed_rows ? p.embed_rows - 1 : id);  // never read outside the table
      return p.embed + static_cast<size_t>(id) * p.k;
    }
    return p.x + static_cast<size_t>(m) * p.k;
  };
  if (embed && blockIdx.x == 0 && p.hidden_out) {  // the residual stream of layer 0
    for (int i = tid; i < M * p.k; i += blockDim.x) {
      const int r = i / p.k, k = i % p.k;
      p.hidden_out[static_cast<size_t>(r) * p.k + k] = f_to_bf16_bits(bf(u16_to_f(row_src(r)[k]) * p.emb_mult));
    }
  }
  if (p.pro != PRO_NONE) {  // RMSNorm statistics: full-row sum of squares, warps combined in a fixed order
    for (int m = 0; m < M; ++m) {
      const uint16_t* src = row_src(m);
      float ss = 0.f;
      for (int k = lane * 8; k < Kw; k += 256) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(src + k0 + k), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float h = embed ? bf(f[e] * p.emb_mult) : f[e];  // embed_tokens(ids) * 12 (llm_mega.py:514)
          ss += h * h;
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) s_ss[warp * 8 + m] = ss;
    }
    __syncthreads();
  }
  for (int m = 0; m < M; ++m) {
    const uint16_t* src = row_src(m);
    float rstd = 1.f;
    if (p.pro != PRO_NONE) {
      float tsum = 0.f;
      for (int q = 0; q < W; ++q) tsum += s_ss[q * 8 + m];
      rstd = 1.f / sqrtf(tsum / static_cast<float>(p.k) + p.eps);
    }
    float am = 0.f;
    for (int k = lane * 8; k < Kw; k += 256) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(src + k0 + k), f);
      if (p.pro != PRO_NONE) {
        float wn[8];
        unpack8(*reinterpret_cast<const uint4*>(p.norm_w + k0 + k), wn);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float h = embed ? bf(f[e] * p.emb_mult) : f[e];
          f[e] = bf(wn[e] * bf(h * rstd));  // weight * bf16(x * rstd)  (modeling_granite.py:192-197)
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(f[e]));
      *reinterpret_cast<uint4*>(xw + m * xstride + k) = pack8(f);
    }
    int shift = 0;
    if (FMT != SB_FMT_BF16) {  // -> f16 scaled by a power of two per (warp, row): exact
      am = warp_max(am);
      int e2 = 0;
      if (am > 0.f) frexpf(am, &e2);
      shift = 15 - e2;  // slice max * 2^shift in [2^14, 2^15)
      for (int k = lane * 8; k < Kw; k += 256) {  // same lane wrote these elements
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(xw + m * xstride + k), f);
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __half2 hh = __floats2half2_rn(ldexpf(f[2 * e], shift), ldexpf(f[2 * e + 1], shift));
          h[e] = *reinterpret_cast<uint32_t*>(&hh);
        }
        *reinterpret_cast<uint4*>(xw + m * xstride + k) = make_uint4(h[0], h[1], h[2], h[3]);
      }
    }
    if (lane == 0) s_shift[warp * 8 + m] = shift;
  }
  __syncwarp();
  // D-fragment column j is token j: this lane's columns 2c and 2c+1
  const int sh0 = s_shift[warp * 8 + min(2 * c, M - 1)];
  const int sh1 = s_shift[warp * 8 + min(2 * c + 1, M - 1)];
  const uint16_t* xb = xw + (g < M ? g : M - 1) * xstride + 2 * c;  // B fragment base of this lane

  // ---- 3. tiles: decode from the ring, tensor cores, batched reduction ----------
  for (int jb = 0; jb < ntile; jb += batch) {
    const int nb = min(batch, ntile - jb);
    for (int jj = 0; jj < nb; ++jj) {
      const int j = jb + jj;
      const uint8_t* slot = ring + static_cast<size_t>(j % slots) * slot_bytes;
      ring_wait(bars + (j % slots), static_cast<uint32_t>((j / slots) & 1), err);
      // one kgroup of this warp's K slice into acc (decode + mma.sync chain)
      auto kg_step = [&](int q, float* acc) {
        const int kg = warp * KPW + q;
        const uint4 a = *reinterpret_cast<const uint4*>(slot + static_cast<size_t>(kg) * 512 + lane * 16);
        const uint16_t* xq = xb + q * KGE;
        if constexpr (FMT == SB_FMT_NVFP4) {
          const uint2 s2 = *reinterpret_cast<const uint2*>(slot + wbytes + static_cast<size_t>(kg) * 64 + g * 8);
          const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
          uint32_t sc[4];  // f16x2 {scale(row g), scale(row g+8)} for k-steps 0..3
          e4m3x4_to_h2x2(s2.x, sc[0], sc[1]);
          e4m3x4_to_h2x2(s2.y, sc[2], sc[3]);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            uint32_t A[4];
            e2m1x8_to_h2x4(wv[t], A[0], A[1], A[2], A[3]);
            const uint32_t slo = __byte_perm(sc[t], 0, 0x1010), shi = __byte_perm(sc[t], 0, 0x3232);
            A[0] = hmul2_u32(A[0], slo);
            A[2] = hmul2_u32(A[2], slo);
            A[1] = hmul2_u32(A[1], shi);
            A[3] = hmul2_u32(A[3], shi);
            mma_f16(acc, A, *reinterpret_cast<const uint32_t*>(xq + t * 16),
                    *reinterpret_cast<const uint32_t*>(xq + t * 16 + 8));
          }
        } else if constexpr (FMT == SB_FMT_FP8 || FMT == SB_FMT_INT8) {
          const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            uint32_t A[4];
            if constexpr (FMT == SB_FMT_FP8) {
              e4m3x4_to_h2x2(wv[2 * t], A[0], A[1]);
              e4m3x4_to_h2x2(wv[2 * t + 1], A[2], A[3]);
            } else {
              i8x4_to_h2x2(wv[2 * t], A[0], A[1]);
              i8x4_to_h2x2(wv[2 * t + 1], A[2], A[3]);
            }
            mma_f16(acc, A, *reinterpret_cast<const uint32_t*>(xq + t * 16),
                    *reinterpret_cast<const uint32_t*>(xq + t * 16 + 8));
          }
        } else {
          const uint32_t A[4] = {a.x, a.y, a.z, a.w};
          mma_bf16(acc, A, *reinterpret_cast<const uint32_t*>(xq), *reinterpret_cast<const uint32_t*>(xq + 8));
        }
      };
      // two independent accumulator chains (kgroups in pairs), summed at the end
      float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < KPW; q += 2) {
        kg_step(q, acc);
        kg_step(q + 1, acc2);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] += acc2[e];
      // undo this warp's activation scale, store the partial of tile jj
      float* rw = red + (static_cast<size_t>(jj) * W + warp) * 16 * M;
      const int col = 2 * c;
      if (col < M) {
        rw[g * M + col] = ldexpf(acc[0], -sh0);
        rw[(g + 8) * M + col] = ldexpf(acc[2], -sh0);
      }
      if (col + 1 < M) {
        rw[g * M + col + 1] = ldexpf(acc[1], -sh1);
        rw[(g + 8) * M + col + 1] = ldexpf(acc[3], -sh1);
      }
    }
    __syncthreads();  // all warps done with this batch's slots and partials
    // refill the slots of this batch with the tiles one ring further on
    if (tid == 0)
      for (int jj = 0; jj < nb; ++jj)
        if (jb + jj + slots < ntile) issue_tile(jb + jj + slots);
    // reduce over warps in a fixed order
    for (int i = tid; i < nb * 16 * M; i += blockDim.x) {
      const int jj = i / (16 * M), rm = i % (16 * M);
      float sum = 0.f;
      for (int q = 0; q < W; ++q) sum += red[(static_cast<size_t>(jj) * W + q) * 16 * M + rm];
      tot[i] = sum;
    }
    __syncthreads();
    gemv_epilogue<FMT>(p, tot, (t0 + jb) * 16, nb * 16, M, s_best, s_bval, jb == 0, jb + nb >= ntile, tid,
                       blockDim.x);
    __syncthreads();
  }
  gemv_argmax_finish(p, s_best, s_bval, M, ntile > 0, s_flag);
}

// ---- host side ------------------------------------------------------------------
static const int kSMs = 148;
static const size_t kDecSmem = 220 * 1024;

bool gemv_dec_plan(int fmt, int n_tiles, int k, int m, DecPlan& pl) {
  if (m < 1 || m > 8) return false;
  const int kge = kgroup_elems(fmt);
  const int ksteps = k / 16;
  int ksw = 16;
  if (ksteps % ksw) return false;
  if (ksteps / ksw > 16) ksw = 32;
  if (ksteps % ksw) return false;
  const int W = ksteps / ksw;
  if (W < 1 || W > 16 || (ksw * 16) % kge) return false;
  const size_t wbytes = static_cast<size_t>(k / kge) * 512;
  const size_t sbytes = fmt == SB_FMT_NVFP4 ? static_cast<size_t>(k / 64) * 64 : 0;
  const size_t slot = (wbytes + sbytes + 127) & ~size_t(127);  // = dec_layout().slot_bytes
  // Two CTAs per SM (16 warps per SM on independent tiles) when two rings of
  // <= 88 KiB fit; else one CTA per SM with a deep ring.
  const bool two = 2 * slot <= 88 * 1024 && W <= 8;
  const int cap = two ? 2 * kSMs : kSMs;
  const int n_ctas = n_tiles < cap ? n_tiles : cap;
  const int per = (n_tiles + n_ctas - 1) / n_ctas;
  int slots = static_cast<int>((two ? 88 : 160) * 1024 / slot);
  if (slots == 0 && !two && per == 1 && slot <= 200 * 1024) slots = 1;
  if (slots > 2 * per) slots = 2 * per;
  if (slots > 16) slots = 16;
  // a CTA that owns a single tile loads nothing after it: one slot serves
  // (the [2048 x 8192] down projection in 1-byte formats: 131 KiB tiles)
  if (slots < 2 && !(slots == 1 && per == 1)) return false;
  int batch = slots >= 2 ? slots / 2 : 1;  // >= 1: the tile loop advances by batch
  // reduction buffers: batch * (W + 1) * 16 * m floats
  while (batch > 1 && static_cast<size_t>(batch) * (W + 1) * 16 * m * 4 > 48 * 1024) --batch;
  const size_t smem = dec_layout(wbytes + sbytes, slots, batch, W, m, ksw * 16).total;
  if (smem > (two ? kDecSmem / 2 : kDecSmem)) return false;
  pl.ksw = ksw;
  pl.warps = W;
  pl.slots = slots;
  pl.batch = batch;
  pl.n_ctas = n_ctas;
  pl.smem = smem;
  return true;
}

template <int FMT, int KSW>
static int dec_launch_t(const GemvParams& p, const DecPlan& pl, bool pdl, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  static unsigned configured = 0;
  if (!(configured & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv_dec<FMT, KSW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kDecSmem));
    if (e != cudaSuccess) return e;
    configured |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_ctas);
  cfg.blockDim = dim3(pl.warps * 32);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  note_launch();
  return cudaLaunchKernelEx(&cfg, k_gemv_dec<FMT, KSW>, p, pl.slots, pl.batch);
}

template <int FMT>
static int dec_launch_f(const GemvParams& p, const DecPlan& pl, bool pdl, cudaStream_t s) {
  return pl.ksw == 16 ? dec_launch_t<FMT, 16>(p, pl, pdl, s) : dec_launch_t<FMT, 32>(p, pl, pdl, s);
}

int gemv_dec_launch(const GemvParams& p, const DecPlan& pl, int fmt, bool pdl, cudaStream_t s) {
  switch (fmt) {
    case SB_FMT_BF16: return dec_launch_f<SB_FMT_BF16>(p, pl, pdl, s);
    case SB_FMT_FP8: return dec_launch_f<SB_FMT_FP8>(p, pl, pdl, s);
    case SB_FMT_INT8: return dec_launch_f<SB_FMT_INT8>(p, pl, pdl, s);
    case SB_FMT_NVFP4: return dec_launch_f<SB_FMT_NVFP4>(p, pl, pdl, s);
  }
  return SB_ERR_ARG;
}

}  // namespace sb
