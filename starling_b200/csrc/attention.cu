// Decode / verify attention over the static KV cache, sm_100a.
//
// Replaces the reference's per-layer attention block
// (src/starling/granite/llm_mega.py:549-556 and the HF eager path
// transformers modeling_granite.py:89-112): repeat_kv copies of K/V, a
// scores matmul over all max_cache_len slots, an additive -max mask, an fp32
// softmax cast to bf16 and a probs @ V matmul.  Here:
//  * no repeat_kv: one CTA (or a cluster of `split` CTAs) serves one
//    (stream, KV head) and all of its query heads (and, for verify, all query
//    tokens) at once;
//  * only keys that can be valid are read: the prompt part [0, prompt_len)
//    and the generated part [pad_len, slot + m), skipping the right-padding
//    hole, which is exactly the set the reference's mask leaves at 0 (masked
//    slots contribute exp(-inf) = 0).  Each part is cut into tiles of 64
//    keys; the tiles are shared out over the cluster;
//  * K tiles and then V tiles stream through a ring of shared-memory slots by
//    TMA (cp.async.bulk.tensor, 128-byte swizzle, two 64-dim boxes per tile)
//    completing on mbarriers; the last tile of a part loads only the 32-key
//    boxes that hold its keys (a part over-reads at most 31 keys: DRAM reads
//    1.07x the valid K/V bytes at 48 streams, 1.30x with whole tiles).  Tiles whose keys are all older than this
//    step are issued BEFORE griddepcontrol.wait, so those loads overlap the
//    q/k/v GEMM that precedes the attention;
//  * both contractions run on the tensor cores (mma.sync m16n8k16, bf16 in,
//    fp32 accumulate): scores^T = K . Q^T per tile with ldmatrix from the
//    swizzled tile (conflict-free), then P . V with ldmatrix.trans.  bf16
//    products are exact, so this is the reference's bf16 matmul up to the
//    fp32 summation order;
//  * rounding points follow the reference: score = bf16(bf16(q.k) * scale),
//    p = bf16(exp(s - max) * (1/sum)) in fp32 with the max and sum over ALL
//    keys (combined across the cluster through distributed shared memory in
//    rank order), out = bf16(sum_j p_j v_j).
// Every ring wait is bounded; on expiry the kernel records SB_CTRL_ERR = 3
// and carries on with invalid results instead of hanging.
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include "attention.cuh"
#include "operand.cuh"

namespace cg = cooperative_groups;

namespace sb {

namespace {

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(su32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 2D TMA tile load of one box (64 dims x tile keys) at (x, y) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          su32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __noinline__ void ring_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = gtimer();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return;
    if (gtimer() - t0 > 2000000000ull) {
      if (err) atomicExch(err, 3);
      return;
    }
  }
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// byte offset of (row, 16-byte chunk) in a 128-byte-swizzled box of 128-byte rows
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}



}  // namespace

// Shared-memory layout (offsets from a 1024-byte-aligned base), identical on
// host and device.  cap = keys per CTA at most (a multiple of the tile size tk).
struct AttnLayout {
  size_t ring, bars, qb, sc, outp, wmax, psum, stat, zero, total;
};
__host__ __device__ inline AttnLayout attn_layout(int R, int cap, int slots, int tk) {
  auto up = [](size_t x) { return (x + 15) & ~size_t(15); };
  AttnLayout L;
  L.ring = 0;
  L.bars = static_cast<size_t>(slots) * tk * 256;
  L.qb = up(L.bars + 8 * static_cast<size_t>(slots));
  L.sc = up(L.qb + static_cast<size_t>(R) * 136 * 2);           // q bf16 [R][136]
  L.outp = up(L.sc + static_cast<size_t>(R) * (cap + 8) * 2);   // scores, then p, bf16 [R][cap + 8]
  L.wmax = up(L.outp + static_cast<size_t>(R) * 128 * 4);       // P.V f32 [R][128]
  L.psum = up(L.wmax + 8 * static_cast<size_t>(R) * 4);         // per-warp row max [8][R]
  L.stat = up(L.psum + 8 * static_cast<size_t>(R) * 4);         // per-warp row sum [R][8]
  L.zero = up(L.stat + 2 * static_cast<size_t>(R) * 4);         // max, sum [R]
  L.total = up(L.zero + 16) + 1024;                             // + alignment slack
  return L;
}

// NT = ceil(R / 8) q-row tiles of the score MMA (R = query rows per KV head);
// TK keys per tile (a tile is two swizzled 64-dim boxes of TK * 128 bytes).
template <int NT, int TK>
__global__ void __launch_bounds__(256, 2)
    k_attn(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap tmk,
           const __grid_constant__ CUtensorMap tmv, const __grid_constant__ CUtensorMap tmk32,
           const __grid_constant__ CUtensorMap tmv32) {
  constexpr int MT = (NT + 1) / 2;  // q-row m-tiles of the P.V MMA
  constexpr int kTK = TK;
  constexpr int kTileBytes = TK * 256;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (su32(smem_raw) & 1023)) & 1023);
  const int split = p.split;
  const int rank = split > 1 ? static_cast<int>(cg::this_cluster().block_rank()) : 0;
  // z = stream * qblocks + query block; q / out rows of the block start at z * m_per
  const int kvh = blockIdx.y, zb = blockIdx.z, b = zb / p.qblocks, qblk = zb % p.qblocks;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int G = p.n_q / p.n_kv;
  const int R = G * p.m_per;
  const int cap = p.chunk_cap;
  const int cst = cap + 8;  // score/p row stride (elements): 16 mod 128 bytes -> conflict-free ldmatrix
  const AttnLayout L = attn_layout(R, cap, p.slots, TK);
  uint8_t* ring = smem + L.ring;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint16_t* qb = reinterpret_cast<uint16_t*>(smem + L.qb);
  uint16_t* sc = reinterpret_cast<uint16_t*>(smem + L.sc);
  float* outp = reinterpret_cast<float*>(smem + L.outp);
  float* wmax = reinterpret_cast<float*>(smem + L.wmax);
  float* psum = reinterpret_cast<float*>(smem + L.psum);
  float* smax = reinterpret_cast<float*>(smem + L.stat);
  float* ssum = smax + R;
  uint16_t* zrow = reinterpret_cast<uint16_t*>(smem + L.zero);  // 16 zero bytes
  int32_t* err = p.ctrl + SB_CTRL_ERR;

  // ---- this CTA's tiles (device values that are stable before the wait: the
  // slot and the lengths were written by kernels that precede the q/k/v GEMM)
  const int slot = p.ctrl[SB_CTRL_SLOT] + qblk * p.m_per;
  const int pad_len = p.ctrl[SB_CTRL_PADLEN];
  int kv_len = slot + p.m_per;
  kv_len = kv_len > p.max_len ? p.max_len : kv_len;
  const int plen = p.prompt_len ? p.prompt_len[b] : kv_len;
  if (p.qblocks > 1 && split == 1 && slot >= plen) {
    // prefill: every query of this block is a prompt's padding; its rows are
    // never used (later layers see them only through row-local operations)
    pdl_wait();
    pdl_launch();
    for (int i = tid; i < R * 64; i += blockDim.x) {
      const int r = i >> 6, mi = r / G, gi = r % G;
      const size_t t = static_cast<size_t>(zb) * p.m_per + mi;
      *reinterpret_cast<uint32_t*>(p.out + t * p.n_q * 128 + (kvh * G + gi) * 128 + (i & 63) * 2) = 0u;
    }
    return;
  }
  const int n1 = plen < kv_len ? plen : kv_len;     // prompt part [0, n1)
  const int g0 = plen < pad_len ? pad_len : n1;     // generated part [g0, kv_len)
  const int n2 = kv_len > g0 ? kv_len - g0 : 0;
  const int t1 = (n1 + kTK - 1) / kTK, t2 = (n2 + kTK - 1) / kTK;
  const int per = (t1 + t2 + split - 1) / split;
  const int i0 = rank * per < t1 + t2 ? rank * per : t1 + t2;
  const int nT = (i0 + per < t1 + t2 ? i0 + per : t1 + t2) - i0;  // this CTA's tiles
  const int nk = nT * kTK;                                          // CTA-local key slots
  auto tstart = [&](int u) { const int i = i0 + u; return i < t1 ? kTK * i : g0 + kTK * (i - t1); };
  auto trows = [&](int u) {
    const int i = i0 + u;
    const int e = i < t1 ? n1 : kv_len, s0 = tstart(u);
    return e - s0 < kTK ? e - s0 : kTK;
  };
  const int head_row0 = (b * p.n_kv + kvh) * p.max_len;
  // item it: K tile it (< nT) or V tile it - nT -> slot it % slots.  A full
  // tile is two boxes of TK keys; a part's last tile takes the 32-key boxes
  // that hold its rows (the swizzle pattern repeats every 8 rows, so a box at
  // row 32i lands exactly where the full box would have put those rows).
  auto item_bytes = [&](int it) {
    const int r = trows(it < nT ? it : it - nT);
    return r == kTK ? kTileBytes : (r + 31) / 32 * 32 * 256;
  };
  auto issue = [&](int it) {
    const int u = it < nT ? it : it - nT;
    uint8_t* dst = ring + static_cast<size_t>(it % p.slots) * kTileBytes;
    uint64_t* bar = bars + (it % p.slots);
    const int r = trows(u), y = head_row0 + tstart(u);
    if (r == kTK) {
      const CUtensorMap* tm = it < nT ? &tmk : &tmv;
      tma_load_2d(dst, tm, 0, y, bar);
      tma_load_2d(dst + kTileBytes / 2, tm, 64, y, bar);
    } else {
      const CUtensorMap* tm = it < nT ? &tmk32 : &tmv32;
      for (int i = 0; i * 32 < r; ++i) {
        tma_load_2d(dst + i * 32 * 128, tm, 0, y + 32 * i, bar);
        tma_load_2d(dst + kTileBytes / 2 + i * 32 * 128, tm, 64, y + 32 * i, bar);
      }
    }
  };
  auto fresh = [&](int it) {  // the tile holds a key written by the preceding kernel
    const int u = it < nT ? it : it - nT;
    return tstart(u) + trows(u) > slot;
  };

  const int total = 2 * nT;
  const int first = total < p.slots ? total : p.slots;
  // rows of a slot that a tail tile does not load must hold finite values
  // (its masked scores and zero probabilities cancel them): an older tile's
  // keys / values, or, where the slot's first tile is already a tail, zeros
  bool zeroed = false;
  for (int s0 = 0; s0 < first; ++s0)
    if (item_bytes(s0) < kTileBytes) {
      uint4* z = reinterpret_cast<uint4*>(ring + static_cast<size_t>(s0) * kTileBytes);
      for (int i = tid; i < kTileBytes / 16; i += blockDim.x) z[i] = make_uint4(0u, 0u, 0u, 0u);
      zeroed = true;
    }
  if (zeroed) fence_proxy_async();  // before the tensor copies write the same bytes
  __syncthreads();
  if (tid == 0) {
    for (int s = 0; s < p.slots; ++s) mbar_init(bars + s, 1);
    mbar_fence_init();
    for (int it = 0; it < first; ++it) {
      mbar_expect_tx(bars + it, item_bytes(it));
      if (!fresh(it)) issue(it);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_launch();
  if (tid == 0)
    for (int it = 0; it < first; ++it)
      if (fresh(it)) issue(it);

  // q rows of this KV group (row r = (token mi, head gi)) as bf16
  for (int i = tid; i < R * 64; i += blockDim.x) {
    const int r = i >> 6, d2 = (i & 63) * 2;
    const int mi = r / G, gi = r % G;
    const size_t t = static_cast<size_t>(zb) * p.m_per + mi;
    *reinterpret_cast<uint32_t*>(qb + r * 136 + d2) =
        *reinterpret_cast<const uint32_t*>(p.q + t * p.n_q * 128 + (kvh * G + gi) * 128 + d2);
  }
  if (tid < 4) reinterpret_cast<uint32_t*>(zrow)[tid] = 0u;
  __syncthreads();

  float acc[MT][2][4];  // P.V accumulators [m-tile][n-tile][frag]
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[a][n][e] = 0.f;
  // the q rows this lane's score fragments hold: row n*8 + 2c + h; causal limit slot + token
  int lim[NT][2];
  float lmax[NT][2];  // running max of this lane's scores per row
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = n * 8 + 2 * c + h;
      lim[n][h] = r < R ? slot + r / G : -1;  // -1: padding row, never stored
      lmax[n][h] = -INFINITY;
    }

  // softmax work split: wpr warps per row (R < 8), else one warp per row
  const int wpr = R < 8 ? 8 / R : 1;
  auto softmax = [&]() {
    // row max: lanes sharing c hold the same rows -> reduce over g, then over warps
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float m = lmax[n][h];
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        const int r = n * 8 + 2 * c + h;
        if (g == 0 && r < R) wmax[warp * R + r] = m;
      }
    __syncthreads();
    for (int r = tid; r < R; r += blockDim.x) {
      float m = -INFINITY;
      for (int w = 0; w < 8; ++w) m = fmaxf(m, wmax[w * R + r]);
      smax[r] = m;
    }
    if (split > 1) cg::this_cluster().sync(); else __syncthreads();
    // sum of exp(s - max): (row, part) per warp, 8 keys per lane-step
    for (int r = warp / wpr; r < R && warp < R * wpr; r += (R < 8 ? R : 8)) {
      float gm = -INFINITY;
      for (int q = 0; q < split; ++q)
        gm = fmaxf(gm, split > 1 ? cg::this_cluster().map_shared_rank(smax, q)[r] : smax[r]);
      const int sub = warp % wpr;
      float s = 0.f;
      for (int ch = sub * 32 + lane; ch * 8 < nk; ch += wpr * 32) {
        float f[8];
        unpack8(*reinterpret_cast<const uint4*>(sc + r * cst + ch * 8), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) s += gm == -INFINITY ? 0.f : expf(f[e] - gm);
      }
      s = warp_sum(s);
      if (lane == 0) psum[r * 8 + sub] = s;
      if (lane == 0 && sub == 0) smax[r] = gm;  // the global max, for the normalisation below
    }
    __syncthreads();
    for (int r = tid; r < R; r += blockDim.x) {
      float s = 0.f;
      for (int q = 0; q < wpr; ++q) s += psum[r * 8 + q];
      ssum[r] = s;
    }
    if (split > 1) cg::this_cluster().sync(); else __syncthreads();
    // p = bf16(exp(s - max) * (1/sum)), in place of the scores
    for (int r = warp / wpr; r < R && warp < R * wpr; r += (R < 8 ? R : 8)) {
      float gs = 0.f;
      for (int q = 0; q < split; ++q) gs += split > 1 ? cg::this_cluster().map_shared_rank(ssum, q)[r] : ssum[r];
      const float gm = smax[r], inv = 1.f / gs;
      const int sub = warp % wpr;
      for (int ch = sub * 32 + lane; ch * 8 < nk; ch += wpr * 32) {
        uint4* ptr8 = reinterpret_cast<uint4*>(sc + r * cst + ch * 8);
        float f[8];
        unpack8(*ptr8, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = gm == -INFINITY ? 0.f : expf(f[e] - gm) * inv;  // softmax(..., float32)
        *ptr8 = pack8(f);                                                                  // .to(bf16)
      }
    }
    __syncthreads();
  };

  for (int it = 0; it < total; ++it) {
    if (it == nT) softmax();
    ring_wait(bars + (it % p.slots), static_cast<uint32_t>((it / p.slots) & 1), err);
    const uint32_t tile = su32(ring + static_cast<size_t>(it % p.slots) * kTileBytes);
    if (it < nT) {
      // ---- scores^T[key][row] = K . Q^T: warp w takes keys 16w..16w+15 of the tile
      const int u = it;
      if (warp * 16 < kTK) {
      float d[NT][4];
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) d[n][e] = 0.f;
      const int arow = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
      const int rows = trows(u), k0 = tstart(u);
      if (warp * 16 < rows) {  // warps past the tile's keys only write masked scores
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t a[4];
        ldsm_x4(tile + (ks >> 2) * (kTileBytes / 2) + swz(arow, (ks & 3) * 2 + (lane >> 4)), a);
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const int qr = n * 8 + g;
          uint32_t b0 = 0, b1 = 0;
          if (qr < R) {
            const uint16_t* qp = qb + qr * 136 + ks * 16 + 2 * c;
            b0 = *reinterpret_cast<const uint32_t*>(qp);
            b1 = *reinterpret_cast<const uint32_t*>(qp + 8);
          }
          mma_bf16(d[n], a, b0, b1);
        }
      }
      }
#pragma unroll
      for (int h8 = 0; h8 < 2; ++h8) {
        const int key = warp * 16 + g + h8 * 8;  // key within the tile
        const int pk = key < rows ? k0 + key : 0x7fffffff;
        uint16_t* srow = sc + u * kTK + key;
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            if (lim[n][h] >= 0) {
              const bool ok = pk <= lim[n][h];
              const float sv = ok ? bf(bf(d[n][h8 * 2 + h]) * p.attn_mult) : -INFINITY;
              if (ok) lmax[n][h] = fmaxf(lmax[n][h], sv);
              srow[(n * 8 + 2 * c + h) * cst] = ok ? f_to_bf16_bits(sv) : static_cast<uint16_t>(0xFF80u);
            }
      }
      }
    } else {
      // ---- out[row][dim] += P . V: warp w takes dims 16w..16w+15 (two n-tiles)
      const int u = it - nT;
      const int vrow_l = (lane & 7) + 8 * ((lane >> 3) & 1);
      const int dchunk = warp * 2 + (lane >> 4);  // 8-dim chunk 0..15
#pragma unroll
      for (int ks = 0; ks < kTK / 16; ++ks) {
        uint32_t bv[4];
        ldsm_x4_t(tile + (dchunk >> 3) * (kTileBytes / 2) + swz(ks * 16 + vrow_l, dchunk & 7), bv);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int prow = mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
          const int pkey = u * kTK + ks * 16 + 8 * (lane >> 4);
          const uint16_t* pa = prow < R ? sc + prow * cst + pkey : zrow;
          uint32_t a[4];
          ldsm_x4(su32(pa), a);
          mma_bf16(acc[mt][0], a, bv[0], bv[1]);
          mma_bf16(acc[mt][1], a, bv[2], bv[3]);
        }
      }
    }
    __syncthreads();  // slot it % slots is free
    if (tid == 0 && it + p.slots < total) {
      const int nx = it + p.slots;
      mbar_expect_tx(bars + (nx % p.slots), item_bytes(nx));
      issue(nx);
    }
  }
  if (nT == 0) {  // no keys here: still take part in the cluster's statistics exchange
    for (int r = tid; r < R; r += blockDim.x) {
      smax[r] = -INFINITY;
      ssum[r] = 0.f;
    }
    if (split > 1) {
      cg::this_cluster().sync();
      cg::this_cluster().sync();
    }
    __syncthreads();
  }

  // ---- this CTA's P.V rows -> outp ---------------------------------------------------------
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = mt * 16 + g + (e >> 1) * 8;
        const int dim = warp * 16 + n * 8 + 2 * c + (e & 1);
        if (r < R) outp[r * 128 + dim] = acc[mt][n][e];
      }

  // ---- combine the cluster's partial outputs, round, store -----------------------------
  if (split > 1) cg::this_cluster().sync(); else __syncthreads();
  // o-projection operand: the largest |output| of each token's slice, as the
  // outputs are stored (a slice is G * 128 consecutive i, a multiple of 32,
  // so every warp iteration belongs to one token); float bits of |x| order
  // like the values
  int* s_tmax = reinterpret_cast<int*>(wmax);  // [m_per] (the row-max scratch is free by now)
  const bool opnd8 = p.opnd && p.opnd_fp8;
  if (rank == 0 && opnd8) {
    for (int mi = tid; mi < p.m_per; mi += blockDim.x) s_tmax[mi] = 0;
    __syncthreads();
  }
  // without the o operand every rank of a cluster finishes a slice of the
  // outputs (four at a time); with it rank 0 finishes them all, as it builds
  // the operand from each token's whole slice.  Sums run in rank order either way.
  const bool spread = split > 1 && !p.opnd;
  if (spread) {
    const int n4 = R * 32, per = (n4 + split - 1) / split;
    const int g1 = (rank + 1) * per < n4 ? (rank + 1) * per : n4;
    for (int gi4 = rank * per + tid; gi4 < g1; gi4 += blockDim.x) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int q = 0; q < split; ++q) {
        const float4 v = reinterpret_cast<const float4*>(cg::this_cluster().map_shared_rank(outp, q))[gi4];
        s4.x += v.x;
        s4.y += v.y;
        s4.z += v.z;
        s4.w += v.w;
      }
      const int i = gi4 * 4, r = i >> 7, dd = i & 127;
      const int mi = r / G, gi = r % G;
      const size_t t = static_cast<size_t>(zb) * p.m_per + mi;
      const uint32_t lo = static_cast<uint32_t>(f_to_bf16_bits(s4.x)) | (static_cast<uint32_t>(f_to_bf16_bits(s4.y)) << 16);
      const uint32_t hi = static_cast<uint32_t>(f_to_bf16_bits(s4.z)) | (static_cast<uint32_t>(f_to_bf16_bits(s4.w)) << 16);
      *reinterpret_cast<uint2*>(p.out + t * p.n_q * 128 + (kvh * G + gi) * 128 + dd) = make_uint2(lo, hi);
    }
  } else if (rank == 0) {
    for (int i = tid; i < R * 128; i += blockDim.x) {
      float s = 0.f;
      for (int q = 0; q < split; ++q) s += split > 1 ? cg::this_cluster().map_shared_rank(outp, q)[i] : outp[i];
      const int r = i >> 7, dd = i & 127;
      const int mi = r / G, gi = r % G;
      const size_t t = static_cast<size_t>(zb) * p.m_per + mi;
      p.out[t * p.n_q * 128 + (kvh * G + gi) * 128 + dd] = f_to_bf16_bits(s);
      if (p.opnd) {
        const float v = bf(s);  // the value the o-projection reads (only this thread reads outp[i] here)
        outp[i] = v;
        if (opnd8) {
          const float m = warp_max(fabsf(v));
          if (lane == 0) atomicMax(s_tmax + mi, __float_as_int(m));
        }
      }
    }
  }
  if (split > 1) cg::this_cluster().sync();
  if (rank == 0 && p.opnd) {
    // this (stream, KV head)'s output slice -- columns kvh * G * 128 .. of each
    // of its m_per tokens -- as the o-projection's operand, one 16-byte chunk
    // per thread
    __syncthreads();
    const size_t kb_bytes = static_cast<size_t>(p.opnd_np) * 128;
    const int slice = G * 128;  // elements of the slice (one K-split rank of the o GEMM)
    const int per = opnd8 ? slice / 16 : slice / 8;  // chunks per token
    for (int j = tid; j < p.m_per * per; j += blockDim.x) {
      const int mi = j / per, cj = j % per;
      const int t = zb * p.m_per + mi;
      const float* row = outp + static_cast<size_t>(mi) * slice;  // rows mi*G .. mi*G+G-1, contiguous
      if (opnd8) {
        const int shift = tc_fp8_shift(__int_as_float(s_tmax[mi]));
        uint4 w0, w1;
        e4m3_split16(row + cj * 16, shift, w0, w1);
        const int c = kvh * per + cj;  // 16-byte chunk of e4m3 along K
        *reinterpret_cast<uint4*>(p.opnd + tc_operand_offset(kb_bytes, t, c)) = w0;
        *reinterpret_cast<uint4*>(p.opnd + tc_operand_offset(kb_bytes, p.opnd_mp + t, c)) = w1;
        if (cj == 0) p.opnd_shift[kvh * p.opnd_mp + t] = shift;
      } else {
        const int c = kvh * per + cj;  // 16-byte chunk of bf16 along K
        *reinterpret_cast<uint4*>(p.opnd + tc_operand_offset(kb_bytes, t, c)) = pack8(row + cj * 8);
      }
    }
  }
}

// ---- host side ------------------------------------------------------------------
int attn_tile_keys(int split) { return split > 1 ? 64 : 128; }

size_t attn_smem_bytes(int R, int chunk_cap, int slots, int tk) { return attn_layout(R, chunk_cap, slots, tk).total; }

int attn_key_capacity(int max_len, int split) {
  const int tk = attn_tile_keys(split);
  const int tiles = (max_len + tk - 1) / tk + 1;  // the padding hole can cut one tile in two
  return (tiles + split - 1) / split * tk;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// [rows][128] bf16 cache viewed as a 2D tensor; box {64 dims, tk keys}, 128B swizzle.
static int cache_map(CUtensorMap* tm, const uint16_t* base, long long rows, int tk) {
  auto fn = encode_fn();
  if (!fn) return SB_ERR_CONFIG;
  cuuint64_t dims[2] = {128, static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(tk)};  // 128 B x tk keys
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : SB_ERR_CONFIG;
}

int attn_launch(const AttnParams& p, int batch, bool pdl, cudaStream_t stream) {
  const int R = (p.n_q / p.n_kv) * p.m_per;
  const int tk = attn_tile_keys(p.split);
  if (R > 64 || R < 1 || p.split < 1 || p.split > 8 || p.slots < 2 || p.chunk_cap % tk) return SB_ERR_CONFIG;
  const size_t smem = attn_smem_bytes(R, p.chunk_cap, p.slots, tk);
  if (smem > 200 * 1024) return SB_ERR_CONFIG;
  CUtensorMap tmk, tmv, tmk32, tmv32;
  if (cache_map(&tmk, p.k_cache, p.cache_rows, tk) || cache_map(&tmv, p.v_cache, p.cache_rows, tk) ||
      cache_map(&tmk32, p.k_cache, p.cache_rows, 32) || cache_map(&tmv32, p.v_cache, p.cache_rows, 32))
    return SB_ERR_CONFIG;
  const int NT = (R + 7) / 8;
  void (*kern)(AttnParams, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap) = nullptr;
  if (tk == 64) {
    switch (NT) {
      case 1: kern = k_attn<1, 64>; break;
      case 2: kern = k_attn<2, 64>; break;
      case 3: kern = k_attn<3, 64>; break;
      case 4: kern = k_attn<4, 64>; break;
      case 5: kern = k_attn<5, 64>; break;
      case 6: kern = k_attn<6, 64>; break;
      case 7: kern = k_attn<7, 64>; break;
      default: kern = k_attn<8, 64>; break;
    }
  } else {
    switch (NT) {
      case 1: kern = k_attn<1, 128>; break;
      case 2: kern = k_attn<2, 128>; break;
      case 3: kern = k_attn<3, 128>; break;
      case 4: kern = k_attn<4, 128>; break;
      case 5: kern = k_attn<5, 128>; break;
      case 6: kern = k_attn<6, 128>; break;
      case 7: kern = k_attn<7, 128>; break;
      default: kern = k_attn<8, 128>; break;
    }
  }
  int dev = 0;
  cudaGetDevice(&dev);
  static unsigned configured[16] = {};
  const int ki = (NT - 1) + (tk == 64 ? 0 : 8);
  if (!(configured[ki] & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    configured[ki] |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.split, p.n_kv, batch * p.qblocks);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (p.split > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = p.split;
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
  return cudaLaunchKernelEx(&cfg, kern, p, tmk, tmv, tmk32, tmv32);
}

}  // namespace sb
