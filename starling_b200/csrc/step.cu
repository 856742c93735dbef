// Fused decode step for up to 8 token rows, sm_100a: one cooperative launch
// runs a whole forward of sb_decode_step -- every layer's q/k/v, attention,
// o, gate/up and down and the lm_head argmax -- with no kernel boundary and no
// grid barrier: each phase hands its output to the next as epoch-tagged words.
//
//  * one CTA per SM (cooperative launch: all CTAs resident), 16 consumer
//    warps and one producer warp;
//  * the producer warp streams the CTA's share of every weight of the step
//    (layer by layer, projection by projection, then lm_head) into a byte
//    ring of shared memory: bulk copies (cp.async.bulk) completing on "full"
//    mbarriers.  Consumer warps release each ring entry on an "empty"
//    mbarrier as soon as they have read it, so the weight stream runs ahead
//    across projection and layer boundaries and is not held by the grid
//    barriers;
//  * projections: a tile is 16 packed rows (pack.py layout); warp w owns one
//    K slice of a tile (small K: two tiles per round, 8 warps each).  The
//    activation rows are read once per projection straight into mma
//    B-fragment registers, with the RMSNorm / embedding prologue fused and the
//    same per-(warp, row) power-of-two f16 scaling as the decode GEMV; weights
//    are decoded from the ring into mma.m16n8k16 A-fragments exactly as in
//    gemv_dec.cu; per-tile partials are reduced over the warps of the tile in
//    a fixed order; the epilogues are the GEMV's (gemv_epi.cuh);
//  * attention: one CTA per (stream, KV head, key split).  Each split writes
//    its per-row score max and exp-sum to global memory; after a counter wait
//    over the head's splits every split forms the reference's
//    p = bf16(exp(s - max) * (1/sum)) with the global max and sum, writes its
//    partial P.V, and the last split of the head to finish adds the partials
//    in split order and rounds once;
//  * hand-over: every activation another CTA reads (q, this forward's k/v
//    rows, attention output, residual stream, SwiGLU output) is written as
//    8-byte words {two bf16, epoch}, epochs unique per (launch, layer, phase);
//    the reader polls the words it needs.  A buffer is rewritten only one
//    layer later, after every reader of it has fed the all-to-all chain
//    q/k/v -> attention -> o -> gate/up -> down that the writer depends on;
//  * lm_head: each CTA keeps a running (value, index) best per token; the last
//    CTA to finish reduces them (value desc, index asc), applies the decode /
//    verify feedback, resets the counters and advances the sequence number
//    for the next launch.
// Every wait (ring mbarriers, handed-over words, attention counters) is
// bounded in time; on expiry the kernel records SB_CTRL_ERR = 4, every later
// wait returns at once, and the forward's results are invalid.
#include <cstdlib>

#include "gemv_epi.cuh"
#include "step.cuh"

namespace sb {

namespace {

constexpr int kCW = 16;                  // consumer warps
constexpr int kThreads = (kCW + 1) * 32;  // + the producer warp
constexpr int kNBar = 32;                // ring entries in flight at most
constexpr uint32_t kEntryMax = 32 * 1024;
constexpr uint64_t kWaitNs = 1000000000ull;  // bound of every wait (1 s)
constexpr int kErrStep = 4;

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
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
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   su32(dst)),
               "l"(src), "r"(bytes), "r"(su32(bar))
               : "memory");
}
__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned atom_release_add(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ bool aborted(const int32_t* err) { return *reinterpret_cast<const volatile int32_t*>(err) != 0; }
__device__ __forceinline__ void fail_wait(int32_t* err) { atomicCAS(err, 0, kErrStep); }

// Bounded mbarrier wait; false when it expired or another wait already did.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int32_t* err) {
  if (mbar_try_wait(b, parity)) return true;
  const uint64_t t0 = gtime();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(b, parity)) return true;
    if ((it & 63) == 0) {
      if (aborted(err)) return false;
      if (gtime() - t0 > kWaitNs) {
        fail_wait(err);
        return false;
      }
    }
  }
}
// Bounded wait that ignores the abort flag: for copies still in flight into
// this CTA's shared memory, which must land before the CTA exits.
__device__ __forceinline__ bool mbar_drain(uint64_t* b, uint32_t parity, int32_t* err) {
  const uint64_t t0 = gtime();
  while (!mbar_try_wait(b, parity))
    if (gtime() - t0 > kWaitNs) {
      fail_wait(err);
      return false;
    }
  return true;
}
// Bounded wait for *c >= target (wrap-safe).
__device__ __forceinline__ bool counter_wait(const unsigned* c, unsigned target, int32_t* err) {
  const uint64_t t0 = gtime();
  for (uint32_t it = 0;; ++it) {
    if (static_cast<int>(ld_acquire(c) - target) >= 0) return true;
    if ((it & 15) == 15) {
      if (aborted(err)) return false;
      if (gtime() - t0 > kWaitNs) {
        fail_wait(err);
        return false;
      }
    }
  }
}

// the 16 consumer warps only (the producer warp never joins)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }

// ---- handed-over activations: 8-byte words {2 bf16 (low), epoch (high)} ----------
// A word is written and read whole (single-copy atomic), so a reader that sees
// its epoch sees that word's data; no barrier orders writer and reader.
// Epochs are unique per (launch, layer, phase) and never 0 (zeroed buffers).
enum { LL_QKV = 0, LL_ATTN = 1, LL_H_O = 2, LL_ACT = 3, LL_H_DOWN = 4 };
__device__ __forceinline__ unsigned ll_epoch(unsigned seq, int layer, int phase) {
  return (seq * 64u + static_cast<unsigned>(layer)) * 8u + static_cast<unsigned>(phase) + 1u;
}
__device__ __forceinline__ void ll_put(unsigned long long* p, uint32_t data, unsigned epoch) {
  const unsigned long long v = (static_cast<unsigned long long>(epoch) << 32) | data;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ll_ld(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// N words p[0..N) carrying `epoch`: their data (bounded wait)
template <int N>
__device__ __forceinline__ void ll_get(const unsigned long long* p, unsigned epoch, uint32_t* out, int32_t* err) {
  unsigned long long v[N];
#pragma unroll
  for (int i = 0; i < N; ++i) v[i] = ll_ld(p + i);
  bool ok = true;
#pragma unroll
  for (int i = 0; i < N; ++i) ok = ok && static_cast<unsigned>(v[i] >> 32) == epoch;
  if (!ok) {
    const uint64_t t0 = gtime();
    for (uint32_t it = 0; !ok; ++it) {
      ok = true;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        if (static_cast<unsigned>(v[i] >> 32) != epoch) v[i] = ll_ld(p + i);
        ok = ok && static_cast<unsigned>(v[i] >> 32) == epoch;
      }
      if (!ok && (it & 15) == 15 && (aborted(err) || gtime() - t0 > kWaitNs)) {
        if (!aborted(err)) fail_wait(err);
        break;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < N; ++i) out[i] = static_cast<uint32_t>(v[i]);
}
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
  return static_cast<uint32_t>(f_to_bf16_bits(a)) | (static_cast<uint32_t>(f_to_bf16_bits(b)) << 16);
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

constexpr int chunks_for(uint32_t round_bytes) {
  int n = 1;
  while (n < kCW && round_bytes / n > kEntryMax) n *= 2;
  return n;
}

// Work geometry of one projection with K inputs.  A kgroup is KGE K elements
// (512 packed bytes per tile, + 64 scale bytes for NVFP4); a warp slice is
// KPW kgroups of one tile; a round is 16 slices (NG tiles of WT slices); a
// ring entry is SPC consecutive slices of a round (NCH entries per round),
// contiguous in the packed weight and scale arrays.
template <int FMT, int K>
struct Geo {
  static constexpr int KGE = KG<FMT>::E;
  static constexpr int KGT = K / KGE;
  static constexpr int KPW = KGT >= kCW ? KGT / kCW : 1;
  static constexpr int WT = KGT / KPW;
  static constexpr int NG = kCW / WT;
  static constexpr uint32_t SW = KPW * 512u;
  static constexpr uint32_t SS = FMT == SB_FMT_NVFP4 ? KPW * 64u : 0u;
  static constexpr int NCH = chunks_for(kCW * (SW + SS));
  static constexpr int SPC = kCW / NCH;
  static_assert(K % KGE == 0 && KGT % KPW == 0 && kCW % WT == 0 && NG <= 2, "unsupported K");
};

__device__ __forceinline__ void tile_range(int n_tiles, int& t0, int& nt) {
  const int nct = gridDim.x, c = blockIdx.x;
  const int base = n_tiles / nct, extra = n_tiles % nct;
  nt = base + (c < extra ? 1 : 0);
  t0 = c * base + (c < extra ? c : extra);
}

// ---- the weight stream: ring placement ----------------------------------------------
// Entries are placed back to back in the ring; an entry that would cross the
// end starts again at offset 0.  Producer and consumers walk the same entry
// sequence and compute the same placements.
struct RingPos {
  uint32_t phys;  // offset of the next placement
  uint32_t voff;  // running byte count (skips included), for the producer's space check
  int ei;         // entry index
};
__device__ __forceinline__ uint32_t ring_place(RingPos& rp, uint32_t size, uint32_t ring) {
  if (rp.phys + size > ring) {
    rp.voff += ring - rp.phys;
    rp.phys = 0;
  }
  const uint32_t start = rp.phys;
  rp.phys += size;
  rp.voff += size;
  return start;
}

// Keys of one attention unit (stream b, KV head h, split s of n_split): valid
// keys as in attention.cu -- the prompt part [0, n1) and the generated part
// [g0, kv_len) -- numbered 0..nkeys-1; the unit takes ordinals [ka, ka + nk).
struct AttnUnit {
  bool active;
  int b, h, s, bh;
  int n1, g0, kv_len, ka, nk;
  __device__ __forceinline__ int pos(int o) const { return o < n1 ? o : g0 + (o - n1); }
};
__device__ __forceinline__ AttnUnit attn_unit(const StepParams& P, int slot, int pad_len) {
  AttnUnit u;
  const int NS = P.n_split;
  const int c = blockIdx.x;
  u.active = c < P.batch * P.n_kv * NS;
  if (!u.active) return u;
  u.b = c / (P.n_kv * NS);
  u.h = (c / NS) % P.n_kv;
  u.s = c % NS;
  u.bh = u.b * P.n_kv + u.h;
  int kv_len = slot + P.m_per;
  u.kv_len = kv_len > P.max_len ? P.max_len : kv_len;
  const int plen = P.prompt_len ? P.prompt_len[u.b] : u.kv_len;
  u.n1 = plen < u.kv_len ? plen : u.kv_len;
  u.g0 = plen < pad_len ? pad_len : u.n1;
  const int n2 = u.kv_len > u.g0 ? u.kv_len - u.g0 : 0;
  const int nkeys = u.n1 + n2;
  u.ka = u.s * nkeys / NS;
  u.nk = (u.s + 1) * nkeys / NS - u.ka;  // <= kStepKeys (host plan)
  return u;
}
__device__ __forceinline__ uint32_t kv_entry_bytes(int nk) { return (static_cast<uint32_t>(nk) * 512u + 127u) & ~127u; }

// ---- producer ---------------------------------------------------------------------
struct Prod {
  uint8_t* ring;
  uint32_t ring_bytes;
  uint64_t* full;
  uint64_t* empty;
  uint32_t* endv;
  uint32_t* txv;     // bytes in flight of each entry
  int32_t* err;
  RingPos rp;
  uint32_t rel_end;
  int rel;
  int landed;        // entries before this one have landed
  uint32_t inflight;  // bytes issued and not yet landed
  uint32_t cap;       // at most this many bytes in flight (queueing in front of the step's own loads)
  bool stop;          // a wait failed: issue nothing more
};

// Place the next entry (size bytes, tx bytes will land in it): wait until its
// ring bytes and its mbarrier are free, arm the full barrier.  Returns its
// shared-memory address, or null once a wait has failed (nothing more is
// issued: a full barrier is armed again only after its previous phase is
// seen complete, never over an unfinished one).
__device__ __forceinline__ uint8_t* prod_begin(Prod& pr, uint32_t size, uint32_t tx) {
  if (pr.stop) return nullptr;
  const int ei = pr.rp.ei;
  const uint32_t start = ring_place(pr.rp, size, pr.ring_bytes);
  const uint32_t vend = pr.rp.voff;  // virtual end of this entry
  while (pr.rel < ei && (vend > pr.rel_end + pr.ring_bytes || ei - pr.rel >= kNBar)) {
    if (!mbar_wait(pr.empty + pr.rel % kNBar, static_cast<uint32_t>((pr.rel / kNBar) & 1), pr.err)) {
      pr.stop = true;
      return nullptr;
    }
    pr.rel_end = pr.endv[pr.rel % kNBar];
    ++pr.rel;
  }
  while (pr.landed < pr.rel) pr.inflight -= pr.txv[pr.landed++ % kNBar];  // released => landed
  while (pr.landed < ei && pr.inflight + tx > pr.cap) {
    if (!mbar_wait(pr.full + pr.landed % kNBar, static_cast<uint32_t>((pr.landed / kNBar) & 1), pr.err)) {
      pr.stop = true;
      return nullptr;
    }
    pr.inflight -= pr.txv[pr.landed++ % kNBar];
  }
  if (ei >= kNBar && !mbar_try_wait(pr.full + ei % kNBar, static_cast<uint32_t>(((ei - kNBar) / kNBar) & 1))) {
    pr.stop = true;  // the slot's previous entry has not landed (only after a failed wait elsewhere)
    return nullptr;
  }
  mbar_expect_tx(pr.full + ei % kNBar, tx);
  pr.endv[ei % kNBar] = vend;
  pr.txv[ei % kNBar] = tx;
  pr.inflight += tx;
  ++pr.rp.ei;
  return pr.ring + start;
}
__device__ __forceinline__ void prod_copy(Prod& pr, uint8_t* dst, const void* src, uint32_t bytes) {
  uint64_t* fb = pr.full + (pr.rp.ei - 1) % kNBar;
  const uint8_t* s8 = static_cast<const uint8_t*>(src);
  for (uint32_t o = 0; o < bytes; o += 32768u) bulk_g2s(dst + o, s8 + o, min(32768u, bytes - o), fb);
}

template <int FMT, int K>
__device__ void produce(Prod& pr, const uint8_t* w, const uint8_t* s, int n_tiles) {
  using G = Geo<FMT, K>;
  int t0, nt;
  tile_range(n_tiles, t0, nt);
  const int S0 = t0 * G::WT, S1 = (t0 + nt) * G::WT;
  for (int ra = S0; ra < S1; ra += kCW)
    for (int ch = 0; ch < G::NCH; ++ch) {
      const int ea = ra + ch * G::SPC;
      if (ea >= S1) break;
      const int nsl = min(G::SPC, S1 - ea);
      const uint32_t wb = nsl * G::SW, sb = nsl * G::SS;
      uint8_t* dst = prod_begin(pr, (wb + sb + 127u) & ~127u, wb + sb);
      if (!dst) return;
      prod_copy(pr, dst, w + static_cast<size_t>(ea) * G::SW, wb);
      if (sb) prod_copy(pr, dst + wb, s + static_cast<size_t>(ea) * G::SS, sb);
    }
}
// a small constant vector (RMSNorm weights): one entry
__device__ __forceinline__ void produce_vec(Prod& pr, const uint16_t* v, int n) {
  const uint32_t bytes = static_cast<uint32_t>(n) * 2u;
  uint8_t* dst = prod_begin(pr, (bytes + 127u) & ~127u, bytes);
  if (dst) prod_copy(pr, dst, v, bytes);
}
// the attention unit's K and V rows written before this forward: K rows
// [0, nk) then V rows, 256 bytes each (rows of this forward's tokens are
// filled in by the consumers after the q/k/v phase)
__device__ __forceinline__ void produce_kv(Prod& pr, const StepParams& P, const AttnUnit& u, const StepLayer& L,
                                           int slot) {
  auto old_run = [&](int o0, int o1, int& p0) {  // ordinals [o0, o1) -> positions p0.. (contiguous), old keys only
    p0 = u.pos(o0);
    int cnt = o1 - o0;
    if (p0 + cnt > slot) cnt = slot > p0 ? slot - p0 : 0;
    return cnt;
  };
  const int e1 = min(u.ka + u.nk, u.n1);  // ordinals in the prompt part: [ka, e1)
  int pa = 0, pb = 0, ca = 0, cb = 0;
  if (e1 > u.ka) ca = old_run(u.ka, e1, pa);
  const int o2 = max(u.ka, u.n1);
  if (u.ka + u.nk > o2) cb = old_run(o2, u.ka + u.nk, pb);
  const uint32_t tx = static_cast<uint32_t>(ca + cb) * 512u;
  uint8_t* dst = prod_begin(pr, kv_entry_bytes(u.nk), tx);
  if (!dst) return;
  const size_t row0 = static_cast<size_t>(u.bh) * P.max_len;
  if (ca) {
    prod_copy(pr, dst, L.k_cache + (row0 + pa) * 128, ca * 256u);
    prod_copy(pr, dst + u.nk * 256, L.v_cache + (row0 + pa) * 128, ca * 256u);
  }
  if (cb) {
    const int off = o2 - u.ka;
    prod_copy(pr, dst + off * 256, L.k_cache + (row0 + pb) * 128, cb * 256u);
    prod_copy(pr, dst + u.nk * 256 + off * 256, L.v_cache + (row0 + pb) * 128, cb * 256u);
  }
}

// ---- consumers ----------------------------------------------------------------------
struct Cx {
  uint8_t* ring;
  uint32_t ring_bytes;
  uint64_t* full;
  uint64_t* empty;
  float* red;
  float* tot;
  float* s_ss;
  int* s_shift;
  uint16_t* xs;
  int* s_best;
  float* s_bval;
  int* s_flag;
  GemvParams* sp;
  uint32_t* aq;
  float* asc;
  int32_t* err;
  int tid, warp, lane, M, nb;
  RingPos rp;
  unsigned nbar;
  int slot, pad_len;
};

// next ring entry (size bytes): wait until it has landed
__device__ __forceinline__ const uint8_t* ent_get(const Cx& cx, RingPos& rp, uint32_t size) {
  const uint32_t start = ring_place(rp, size, cx.ring_bytes);
  mbar_wait(cx.full + rp.ei % kNBar, static_cast<uint32_t>((rp.ei / kNBar) & 1), cx.err);
  return cx.ring + start;
}
// this warp is done with the entry ent_get returned last
__device__ __forceinline__ void ent_put(const Cx& cx, RingPos& rp) {
  __syncwarp();
  if (cx.lane == 0) mbar_arrive(cx.empty + rp.ei % kNBar);
  ++rp.ei;
}


// Activation rows -> f16 slices in shared memory (bf16 for bf16 weights):
// warp w < WT converts K slice w of every token into xs[w][m][kw + 8], with
// the RMSNorm / embedding prologue and a power-of-two scale per (slice,
// token) so that the slice maximum lands in [2^14, 2^15) (the decode GEMV's
// scheme); the scales go to s_shift[w][m].  With a prologue, the RMSNorm
// weights are the next ring entry.  Ends with a consumer barrier.
template <int FMT, int K>
__device__ __forceinline__ void load_act(const StepParams& P, const Cx& cx, RingPos& rp, int pro,
                                         const unsigned long long* ll, unsigned epoch) {
  using G = Geo<FMT, K>;
  constexpr int KW = G::KPW * G::KGE;  // K elements per slice
  constexpr int XS = KW + 8;           // row stride (elements)
  constexpr int CPR = KW / 8;          // 16-byte chunks per slice row
  const int lane = cx.lane, warp = cx.warp, M = cx.M;
  const bool embed = pro == PRO_EMBED;
  const int k0 = warp * KW;
  uint16_t* xw = cx.xs + static_cast<size_t>(warp) * M * XS;
  auto row_src = [&](int m) -> const uint16_t* {
    if (embed) {
      int64_t id = P.ids[m];
      id = id < 0 ? 0 : (id >= P.vocab ? P.vocab - 1 : id);  // never read outside the table
      return P.embed + static_cast<size_t>(id) * K;
    }
    return nullptr;
  };
  if (warp < G::WT) {
    // raw rows (embedding scaled: embed_tokens(ids) * 12, llm_mega.py:514); all loads in flight together
#pragma unroll 4
    for (int i = lane; i < M * CPR; i += 32) {
      const int m = i / CPR, k = (i % CPR) * 8;
      uint4 v;
      if (embed) {
        v = __ldg(reinterpret_cast<const uint4*>(row_src(m) + k0 + k));
      } else {  // written by other CTAs in this launch: poll the words
        uint32_t w[4];
        ll_get<4>(ll + static_cast<size_t>(m) * (K / 2) + (k0 + k) / 2, epoch, w, cx.err);
        v = make_uint4(w[0], w[1], w[2], w[3]);
      }
      if (embed) {
        float f[8];
        unpack8(v, f);
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = bf(f[e] * P.emb_mult);
        v = pack8(f);
      }
      *reinterpret_cast<uint4*>(xw + m * XS + k) = v;
    }
    __syncwarp();
    if (pro != PRO_NONE)  // RMSNorm statistics of this slice
      for (int m = 0; m < M; ++m) {
        float ss = 0.f;
        for (int k = lane * 8; k < KW; k += 256) {
          float f[8];
          unpack8(*reinterpret_cast<const uint4*>(xw + m * XS + k), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
        }
        ss = warp_sum(ss);
        if (lane == 0) cx.s_ss[warp * 8 + m] = ss;
      }
  }
  const uint16_t* norm_w = nullptr;
  if (pro != PRO_NONE) norm_w = reinterpret_cast<const uint16_t*>(ent_get(cx, rp, (K * 2u + 127u) & ~127u));
  csync();
  if (warp < G::WT) {
    for (int m = 0; m < M; ++m) {
      float rstd = 1.f;
      if (pro != PRO_NONE) {  // slices of one tile cover K once; fixed-order sum
        float tsum = 0.f;
        for (int q = 0; q < G::WT; ++q) tsum += cx.s_ss[q * 8 + m];
        rstd = 1.f / sqrtf(tsum / static_cast<float>(K) + P.eps);
      }
      float am = 0.f;
      for (int k = lane * 8; k < KW; k += 256) {
        uint4* xp = reinterpret_cast<uint4*>(xw + m * XS + k);
        float f[8];
        unpack8(*xp, f);
        if (pro != PRO_NONE) {
          float wn[8];
          unpack8(*reinterpret_cast<const uint4*>(norm_w + k0 + k), wn);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = bf(wn[e] * bf(f[e] * rstd));  // w * bf16(x * rstd) (modeling_granite.py:192-197)
          *xp = pack8(f);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) am = fmaxf(am, fabsf(f[e]));
      }
      int shift = 0;
      if (FMT != SB_FMT_BF16) {  // -> f16 scaled by a power of two: exact
        am = warp_max(am);
        int e2 = 0;
        if (am > 0.f) frexpf(am, &e2);
        shift = 15 - e2;  // slice max * 2^shift in [2^14, 2^15)
        for (int k = lane * 8; k < KW; k += 256) {  // the lane that wrote these elements
          uint4* xp = reinterpret_cast<uint4*>(xw + m * XS + k);
          float f[8];
          unpack8(*xp, f);
          uint32_t h[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __half2 hh = __floats2half2_rn(ldexpf(f[2 * e], shift), ldexpf(f[2 * e + 1], shift));
            h[e] = *reinterpret_cast<uint32_t*>(&hh);
          }
          *xp = make_uint4(h[0], h[1], h[2], h[3]);
        }
      }
      if (lane == 0) cx.s_shift[warp * 8 + m] = shift;
    }
  }
  if (pro != PRO_NONE) ent_put(cx, rp);
  csync();
}

// One warp slice (KPW kgroups) of a tile into two accumulator chains; xb is
// this lane's B-fragment base in the slice's activation rows.
template <int FMT, int K>
__device__ __forceinline__ void slice_mma(const uint8_t* wsl, const uint8_t* ssl, const uint16_t* xb, float* acc,
                                          float* acc2, int lane) {
  using G = Geo<FMT, K>;
  const int g = lane >> 2;
#pragma unroll
  for (int q = 0; q < G::KPW; ++q) {
    float* d = (q & 1) ? acc2 : acc;
    const uint4 a = *reinterpret_cast<const uint4*>(wsl + q * 512 + lane * 16);
    const uint32_t wv[4] = {a.x, a.y, a.z, a.w};
    const uint16_t* xq = xb + q * G::KGE;
    if constexpr (FMT == SB_FMT_NVFP4) {
      const uint2 s2 = *reinterpret_cast<const uint2*>(ssl + q * 64 + g * 8);
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
        mma_f16(d, A, *reinterpret_cast<const uint32_t*>(xq + t * 16),
                *reinterpret_cast<const uint32_t*>(xq + t * 16 + 8));
      }
    } else if constexpr (FMT == SB_FMT_FP8 || FMT == SB_FMT_INT8) {
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
        mma_f16(d, A, *reinterpret_cast<const uint32_t*>(xq + t * 16),
                *reinterpret_cast<const uint32_t*>(xq + t * 16 + 8));
      }
    } else {
      mma_bf16(d, wv, *reinterpret_cast<const uint32_t*>(xq), *reinterpret_cast<const uint32_t*>(xq + 8));
    }
  }
}

// 2^-s as a float (|s| < 127): the exact power of two
__device__ __forceinline__ float pow2_neg(int s) { return __int_as_float((127 - s) << 23); }

// Epilogues of the fused step: the decode GEMV's operations and rounding
// (gemv_epi.cuh) on rows row0.. of tot, every output another CTA reads
// written as handed-over words with `epoch` (rows in pairs / quads so that a
// word holds two consecutive bf16 outputs).
template <int FMT, int EPI>
__device__ __forceinline__ void step_epi(const StepParams& P, const Cx& cx, const float* tot, int row0, int nrow,
                                         int M, bool first, unsigned epoch) {
  const GemvParams& p = *cx.sp;
  const int tid = cx.tid;
  auto fin = [&](int lrow, int m) -> float {
    float v = tot[lrow * M + m];
    if (FMT == SB_FMT_NVFP4) v *= p.gscale;
    if (FMT == SB_FMT_FP8 || FMT == SB_FMT_INT8) v *= reinterpret_cast<const float*>(p.scale)[row0 + lrow];
    return v;
  };
  if constexpr (EPI == EPI_ARGMAX) {
    gemv_epilogue<FMT, EPI_ARGMAX>(p, tot, row0, nrow, M, cx.s_best, cx.s_bval, first, false, tid, kCW * 32);
  } else if constexpr (EPI == EPI_RESID) {
    // hidden = hidden + bf16(res_mult * bf16(y))   (llm_kernels.py:306-313)
    const int np = nrow / 2;
    for (int i = tid; i < np * M; i += kCW * 32) {
      const int m = i / np, lr = 2 * (i % np), row = row0 + lr;
      if (row >= p.n) continue;
      uint16_t* cp = p.resid_cache + m * p.rc_stride + (row - p.rc_row0);
      const uint32_t w = pack_bf2(u16_to_f(cp[0]) + bf(p.res_mult * bf(fin(lr, m))),
                                  u16_to_f(cp[1]) + bf(p.res_mult * bf(fin(lr + 1, m))));
      *reinterpret_cast<uint32_t*>(cp) = w;
      *reinterpret_cast<uint32_t*>(p.y + static_cast<size_t>(m) * p.n + row) = w;
      ll_put(P.ll_h + static_cast<size_t>(m) * (p.n / 2) + row / 2, w, epoch);
    }
  } else if constexpr (EPI == EPI_SWIGLU) {
    // act = bf16(bf16(silu(gate)) * up)   (llm_kernels.py:252-260); rows gate 2j, up 2j+1
    const int nq = nrow / 4, inter = p.n / 2;
    for (int i = tid; i < nq * M; i += kCW * 32) {
      const int m = i / nq, lr = 4 * (i % nq), row = row0 + lr;
      if (row >= p.n) continue;
      float o[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float gv = bf(fin(lr + 2 * e, m));
        const float sg = bf(gv / (1.f + expf(-gv)));
        o[e] = sg * bf(fin(lr + 2 * e + 1, m));
      }
      ll_put(P.ll_act + static_cast<size_t>(m) * (inter / 2) + row / 4, pack_bf2(o[0], o[1]), epoch);
    }
  } else if constexpr (EPI == EPI_QKV) {
    // q/k: RoPE with each product rounded to bf16 (llm_mega.py:539-543); k/v
    // to cache slot ctrl[SLOT] + token (StaticLayer.update, cache_utils.py:308-335)
    // and, for this forward's attention, to the handed-over words
    const int qk_rows = (p.n_q + p.n_kv) * 128;
    const int nq = nrow / 4;
    for (int i = tid; i < nq * M; i += kCW * 32) {
      const int m = i / nq, lr = 4 * (i % nq), row = row0 + lr;
      if (row >= p.n) continue;
      const int b = m / p.m_per, slot = cx.slot + m % p.m_per;
      const bool slot_ok = slot >= 0 && slot < p.max_len;
      const int head = row >> 7, within = row & 127;
      if (row < qk_rows) {
        const int j = within >> 1;  // rows 2j, 2j+1 -> dims j, j+64; rows 2j+2, 2j+3 -> dims j+1, j+65
        float o1[2], o2[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float x1 = bf(fin(lr + 2 * e, m)), x2 = bf(fin(lr + 2 * e + 1, m));
          const float cs = u16_to_f(p.rope_cache[m * 128 + j + e]);
          const float sn = u16_to_f(p.rope_cache[m * 128 + 64 + j + e]);
          o1[e] = bf(x1 * cs) - bf(x2 * sn);
          o2[e] = bf(x2 * cs) + bf(x1 * sn);
        }
        const uint32_t wlo = pack_bf2(o1[0], o1[1]), whi = pack_bf2(o2[0], o2[1]);
        if (head < p.n_q) {
          unsigned long long* q = P.ll_q + (static_cast<size_t>(m) * p.n_q + head) * 64;
          ll_put(q + j / 2, wlo, epoch);
          ll_put(q + 32 + j / 2, whi, epoch);
        } else {
          const int kh = head - p.n_q;
          if (slot_ok) {
            uint16_t* kc = p.k_cache + ((static_cast<size_t>(b) * p.n_kv + kh) * p.max_len + slot) * 128;
            *reinterpret_cast<uint32_t*>(kc + j) = wlo;
            *reinterpret_cast<uint32_t*>(kc + j + 64) = whi;
          }
          unsigned long long* kv = P.ll_kv + (static_cast<size_t>(m) * p.n_kv + kh) * 128;
          ll_put(kv + j / 2, wlo, epoch);
          ll_put(kv + 32 + j / 2, whi, epoch);
        }
      } else {
        const int vh = head - p.n_q - p.n_kv;  // dims within .. within + 3
        const uint32_t w0 = pack_bf2(fin(lr, m), fin(lr + 1, m)), w1 = pack_bf2(fin(lr + 2, m), fin(lr + 3, m));
        if (slot_ok) {
          uint16_t* vc = p.v_cache + ((static_cast<size_t>(b) * p.n_kv + vh) * p.max_len + slot) * 128 + within;
          *reinterpret_cast<uint32_t*>(vc) = w0;
          *reinterpret_cast<uint32_t*>(vc + 2) = w1;
        }
        unsigned long long* kv = P.ll_kv + (static_cast<size_t>(m) * p.n_kv + vh) * 128 + 64 + within / 2;
        ll_put(kv, w0, epoch);
        ll_put(kv + 1, w1, epoch);
      }
    }
  }
}

// One projection: this CTA's tiles, activation from the handed-over words ll
// (epoch ep_in; pro: prologue), epilogue EPI (compile time) configured in
// *cx.sp writing epoch ep_out.  A CTA without tiles reads nothing.
template <int FMT, int K, int EPI>
__device__ __forceinline__ void gemv_phase(const StepParams& P, Cx& cx, int n_tiles, int pro,
                                           const unsigned long long* ll, unsigned ep_in, unsigned ep_out) {
  using G = Geo<FMT, K>;
  constexpr int XS = G::KPW * G::KGE + 8;
  const int M = cx.M, warp = cx.warp, lane = cx.lane, tid = cx.tid;
  const int g = lane >> 2, c = lane & 3;
  int t0, nt;
  tile_range(n_tiles, t0, nt);
  const int S0 = t0 * G::WT, S1 = (t0 + nt) * G::WT;
  const int rounds = (nt + G::NG - 1) / G::NG;

  RingPos rp = cx.rp;
  if (nt == 0) {  // nothing to compute: only the RMSNorm-weight entry to pass
    if (pro != PRO_NONE) {
      ent_get(cx, rp, (K * 2u + 127u) & ~127u);
      ent_put(cx, rp);
    }
    cx.rp = rp;
    return;
  }
  load_act<FMT, K>(P, cx, rp, pro, ll, ep_in);
  const int sl = warp % G::WT;  // this warp's K slice
  const float us0 = pow2_neg(cx.s_shift[sl * 8 + min(2 * c, M - 1)]);
  const float us1 = pow2_neg(cx.s_shift[sl * 8 + min(2 * c + 1, M - 1)]);
  const uint16_t* xb = cx.xs + (static_cast<size_t>(sl) * M + (g < M ? g : M - 1)) * XS + 2 * c;

  for (int rb = 0; rb < rounds; rb += cx.nb) {
    const int nr = min(cx.nb, rounds - rb);
    for (int r = rb; r < rb + nr; ++r) {
      const int ra = S0 + r * kCW;
      const int gs = ra + warp;  // this warp's slice
      float acc[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ch = 0; ch < G::NCH; ++ch) {
        const int ea = ra + ch * G::SPC;
        if (ea >= S1) break;
        const int nsl = min(G::SPC, S1 - ea);
        const uint8_t* ent = ent_get(cx, rp, (nsl * (G::SW + G::SS) + 127u) & ~127u);
        if (gs >= ea && gs < ea + nsl)
          slice_mma<FMT, K>(ent + (gs - ea) * G::SW, ent + nsl * G::SW + (gs - ea) * G::SS, xb, acc, acc2, lane);
        ent_put(cx, rp);
      }
      if (gs < S1) {  // undo this slice's activation scale, store the partial
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[e] += acc2[e];
        float* rw = cx.red + (static_cast<size_t>(r - rb) * kCW + warp) * 16 * M;
        const int col = 2 * c;
        if (col < M) {
          rw[g * M + col] = acc[0] * us0;
          rw[(g + 8) * M + col] = acc[2] * us0;
        }
        if (col + 1 < M) {
          rw[g * M + col + 1] = acc[1] * us1;
          rw[(g + 8) * M + col + 1] = acc[3] * us1;
        }
      }
    }
    csync();
    // reduce each tile over its WT warps in a fixed order
    const int tile0 = rb * G::NG;
    const int ntl = min(nr * G::NG, nt - tile0);
    for (int i = tid; i < ntl * 16 * M; i += kCW * 32) {
      const int lt = i / (16 * M), rm = i % (16 * M);
      const int r = lt / G::NG, tg = lt % G::NG;
      const float* src = cx.red + (static_cast<size_t>(r) * kCW + tg * G::WT) * 16 * M + rm;
      float sum = 0.f;
      for (int q = 0; q < G::WT; ++q) sum += src[q * 16 * M];
      cx.tot[i] = sum;
    }
    csync();
    step_epi<FMT, EPI>(P, cx, cx.tot, (t0 + tile0) * 16, ntl * 16, M, rb == 0, ep_out);
    csync();
  }
  cx.rp = rp;
}

// Epilogue configuration of one projection (thread 0; read after a csync).
__device__ __forceinline__ void set_epi(const StepParams& P, Cx& cx, int mat, int layer, const uint16_t* rope,
                                        uint16_t* rc) {
  GemvParams* p = cx.sp;
  const bool lm = mat == 4;
  const StepLayer& L = P.layers[lm ? 0 : layer];
  p->scale = lm ? P.lm_s : L.s[mat];
  p->gscale = lm ? P.lm_g : L.g[mat];
  p->n = P.n_rows[mat];
  p->m = cx.M;
  p->ctrl = P.ctrl;
  p->res_mult = P.res_mult;
  if (mat == 0) {
    p->epi = EPI_QKV;
    p->q_out = P.q;
    p->k_cache = L.k_cache;
    p->v_cache = L.v_cache;
    p->n_q = P.n_q;
    p->n_kv = P.n_kv;
    p->max_len = P.max_len;
    p->m_per = P.m_per;
    p->cos_tab = P.cos_tab;
    p->sin_tab = P.sin_tab;
    p->rope_max = P.rope_max;
    p->rope_off = P.rope_off;
    p->rope_cache = rope;
  } else if (mat == 1 || mat == 3) {
    p->epi = EPI_RESID;
    p->y = P.resid;
    p->resid_cache = rc;
    int t0, nt;
    tile_range(P.n_tiles[1], t0, nt);
    p->rc_stride = P.rc_rows;
    p->rc_row0 = t0 * 16;
  } else if (mat == 2) {
    p->epi = EPI_SWIGLU;
    p->y = P.act;
  } else {
    p->epi = EPI_ARGMAX;
    p->logits = P.logits;
    p->logits_mult = P.logits_mult;
  }
}

// Attention of one layer for this CTA's unit.  The K / V rows of older keys
// were streamed into the next ring entry by the producer; rows of this
// forward's tokens are read here (written by the q/k/v phase).
__device__ __forceinline__ void attn_phase(const StepParams& P, Cx& cx, int layer, unsigned ep_in, unsigned ep_out) {
  const AttnUnit u = attn_unit(P, cx.slot, cx.pad_len);
  if (!u.active) return;
  const int NS = P.n_split, G = P.n_q / P.n_kv, R = G * P.m_per;
  const int tid = cx.tid, warp = cx.warp, lane = cx.lane, nk = u.nk;
  const int slot = cx.slot;
  uint8_t* ent = const_cast<uint8_t*>(ent_get(cx, cx.rp, kv_entry_bytes(nk)));
  const uint32_t* kw = reinterpret_cast<const uint32_t*>(ent);          // [nk][64 words]
  const uint16_t* vr = reinterpret_cast<const uint16_t*>(ent + nk * 256);  // [nk][128]

  // q rows (row r = token r / G, query head h*G + r % G) and this forward's K / V
  // rows: handed-over words of the q/k/v phase
  for (int i = tid; i < R * 64; i += kCW * 32) {
    const int r = i >> 6, d2 = i & 63;
    const int mi = r / G, gi = r % G;
    ll_get<1>(P.ll_q + (static_cast<size_t>(u.b * P.m_per + mi) * P.n_q + u.h * G + gi) * 64 + d2, ep_in,
              cx.aq + r * 64 + d2, cx.err);
  }
  for (int i = tid; i < nk * 128; i += kCW * 32) {
    const int j = i >> 7, isv = (i >> 6) & 1, w = i & 63;
    const int ps = u.pos(u.ka + j);
    if (ps < slot) continue;
    const int m = u.b * P.m_per + (ps - slot);
    ll_get<1>(P.ll_kv + (static_cast<size_t>(m) * P.n_kv + u.h) * 128 + isv * 64 + w, ep_in,
              reinterpret_cast<uint32_t*>(ent + (isv ? nk * 256 : 0) + j * 256) + w, cx.err);
  }
  csync();

  // scores, score = bf16(bf16(q.k) * scale).  Eight or more query rows (verify):
  // mma.sync m16n8k16 over (16-row block, 8-key block) tiles, one per warp, the
  // fragments read as 32-bit words of the q and K rows.  Fewer: 4 lanes per
  // (row, key) pair, lane quarter qd taking words qd, qd+4, .. in an order
  // rotated by the key (conflict-free).
  if (R >= 8) {
    const int nrb = (R + 15) / 16, nkb = (nk + 7) / 8, g = lane >> 2, c = lane & 3;
    for (int t = warp; t < nrb * nkb; t += kCW) {
      const int rb = t / nkb, kb = t % nkb;
      const int r0 = rb * 16 + g, r1 = r0 + 8, key = kb * 8 + g;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        uint32_t af[4];
        af[0] = r0 < R ? cx.aq[r0 * 64 + ks * 8 + c] : 0u;
        af[1] = r1 < R ? cx.aq[r1 * 64 + ks * 8 + c] : 0u;
        af[2] = r0 < R ? cx.aq[r0 * 64 + ks * 8 + c + 4] : 0u;
        af[3] = r1 < R ? cx.aq[r1 * 64 + ks * 8 + c + 4] : 0u;
        const uint32_t b0 = key < nk ? kw[key * 64 + ks * 8 + c] : 0u;
        const uint32_t b1 = key < nk ? kw[key * 64 + ks * 8 + c + 4] : 0u;
        mma_bf16(d, af, b0, b1);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e < 2 ? r0 : r1, j = kb * 8 + 2 * c + (e & 1);
        if (r < R && j < nk) {
          const bool valid = u.pos(u.ka + j) <= slot + r / G;  // causal limit slot + token
          cx.asc[r * kStepKeys + j] = valid ? bf(bf(d[e]) * P.attn_mult) : -INFINITY;
        }
      }
    }
  } else
  for (int base = 0; base < R * nk; base += kCW * 8) {
    const int pp = base + warp * 8 + (lane >> 2), qd = lane & 3;
    const bool on = pp < R * nk;
    const int r = on ? pp / nk : 0, j = on ? pp % nk : 0;
    float dot = 0.f;
    if (on) {
      const uint32_t* qr = cx.aq + r * 64;
      const uint32_t* kr = kw + j * 64;
#pragma unroll 8
      for (int it = 0; it < 16; ++it) {
        const int wd = 4 * ((it + j) & 15) + qd;
        const uint32_t qv = qr[wd], kv = kr[wd];
        dot = fmaf(__uint_as_float(qv << 16), __uint_as_float(kv << 16), dot);
        dot = fmaf(__uint_as_float(qv & 0xffff0000u), __uint_as_float(kv & 0xffff0000u), dot);
      }
    }
    dot += __shfl_xor_sync(0xffffffffu, dot, 1);
    dot += __shfl_xor_sync(0xffffffffu, dot, 2);
    if (on && qd == 0) {
      const bool valid = u.pos(u.ka + j) <= slot + r / G;  // causal limit slot + token
      cx.asc[r * kStepKeys + j] = valid ? bf(bf(dot) * P.attn_mult) : -INFINITY;
    }
  }
  csync();
  // per-row max and exp-sum of this split -> global
  float2* stats = P.attn_stats + (static_cast<size_t>(u.bh) * NS) * R;
  for (int r = warp; r < R; r += kCW) {
    const float sv = lane < nk ? cx.asc[r * kStepKeys + lane] : -INFINITY;
    const float mx = warp_max(sv);
    const float l = warp_sum(sv != -INFINITY ? expf(sv - mx) : 0.f);
    if (lane == 0) stats[u.s * R + r] = make_float2(mx, l);
  }
  csync();
  if (tid == 0) {
    red_release_add(P.sync + kSyncStats + u.bh, 1u);
    counter_wait(P.sync + kSyncStats + u.bh, static_cast<unsigned>((layer + 1) * NS), cx.err);
  }
  csync();
  // global max / sum per row over the head's splits (fixed lane order), then p in place
  for (int r = warp; r < R; r += kCW) {
    float2 st = make_float2(-INFINITY, 0.f);
    if (lane < NS) st = __ldcg(stats + lane * R + r);
    const float gm = warp_max(st.x);
    const float gs = warp_sum(st.x == -INFINITY ? 0.f : st.y * expf(st.x - gm));
    const float sv = lane < nk ? cx.asc[r * kStepKeys + lane] : -INFINITY;
    float pj = 0.f;
    if (sv != -INFINITY) pj = bf(expf(sv - gm) * (1.f / gs));  // softmax(..., float32).to(bf16)
    if (lane < nk) cx.asc[r * kStepKeys + lane] = pj;
  }
  csync();
  float* part = P.attn_part + (static_cast<size_t>(u.bh) * NS) * R * 128;
  if (R >= 8) {
    // P.V on mma.sync: one (16-row block, 8-dim block) tile per warp, the
    // probabilities (bf16 values) and V rows packed into fragments, keys past
    // the split's own zero
    const int nrb = (R + 15) / 16, g = lane >> 2, c = lane & 3;
    float* pp = part + static_cast<size_t>(u.s) * R * 128;
    auto pv = [&](int r, int j) { return r < R && j < nk ? cx.asc[r * kStepKeys + j] : 0.f; };
    for (int t = warp; t < nrb * 16; t += kCW) {
      const int rb = t >> 4, db = t & 15;
      const int r0 = rb * 16 + g, r1 = r0 + 8, dim = db * 8 + g;
      auto vv = [&](int j) -> uint32_t { return j < nk ? static_cast<uint32_t>(vr[j * 128 + dim]) : 0u; };
      float d[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ks = 0; ks * 16 < nk; ++ks) {
        const int k0 = ks * 16 + 2 * c;
        uint32_t af[4];
        af[0] = pack_bf2(pv(r0, k0), pv(r0, k0 + 1));
        af[1] = pack_bf2(pv(r1, k0), pv(r1, k0 + 1));
        af[2] = pack_bf2(pv(r0, k0 + 8), pv(r0, k0 + 9));
        af[3] = pack_bf2(pv(r1, k0 + 8), pv(r1, k0 + 9));
        mma_bf16(d, af, vv(k0) | (vv(k0 + 1) << 16), vv(k0 + 8) | (vv(k0 + 9) << 16));
      }
      const int dd = db * 8 + 2 * c;
      if (r0 < R) *reinterpret_cast<float2*>(pp + r0 * 128 + dd) = make_float2(d[0], d[1]);
      if (r1 < R) *reinterpret_cast<float2*>(pp + r1 * 128 + dd) = make_float2(d[2], d[3]);
    }
  } else
  for (int o = tid; o < R * 128; o += kCW * 32) {
    const int r = o >> 7, d = o & 127;
    const float* pr = cx.asc + r * kStepKeys;
    float a0 = 0.f, a1 = 0.f;
    int j = 0;
    for (; j + 1 < nk; j += 2) {
      a0 = fmaf(pr[j], u16_to_f(vr[j * 128 + d]), a0);
      a1 = fmaf(pr[j + 1], u16_to_f(vr[(j + 1) * 128 + d]), a1);
    }
    if (j < nk) a0 = fmaf(pr[j], u16_to_f(vr[j * 128 + d]), a0);
    part[static_cast<size_t>(u.s) * R * 128 + o] = a0 + a1;
  }
  ent_put(cx, cx.rp);
  csync();
  if (tid == 0) {
    const unsigned prev = atom_release_add(P.sync + kSyncCombine + u.bh, 1u);
    *cx.s_flag = prev == static_cast<unsigned>((layer + 1) * NS - 1);
  }
  csync();
  if (*cx.s_flag) {  // last split of this head: sum the partials in split order, round once
    __threadfence();
    for (int o2 = tid; o2 < R * 64; o2 += kCW * 32) {
      const int r = o2 >> 6, o = r * 128 + (o2 & 63) * 2;  // outputs o, o + 1
      float a0 = 0.f, a1 = 0.f;
      for (int q0 = 0; q0 < NS; q0 += 8) {  // 8 loads in flight, summed in split order
        float2 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
          v[q] = q0 + q < NS ? __ldcg(reinterpret_cast<const float2*>(part + static_cast<size_t>(q0 + q) * R * 128 + o))
                             : make_float2(0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          a0 += v[q].x;
          a1 += v[q].y;
        }
      }
      const int mi = r / G, gi = r % G;
      ll_put(P.ll_attn + (static_cast<size_t>(u.b * P.m_per + mi) * P.n_q + u.h * G + gi) * 64 + (o2 & 63),
             pack_bf2(a0, a1), ep_out);
    }
  }
}

// lm_head tail: publish this CTA's best per token; the last CTA reduces all of
// them, applies the decode / verify feedback and resets the counters.
__device__ void lm_finish(const StepParams& P, Cx& cx, bool has_rows) {
  const int tid = cx.tid, lane = cx.lane, warp = cx.warp, M = cx.M;
  const int nct = gridDim.x, cta = blockIdx.x;
  if (tid < M) {
    P.am_val[static_cast<size_t>(cta) * M + tid] = has_rows ? cx.s_bval[tid] : -INFINITY;
    P.am_idx[static_cast<size_t>(cta) * M + tid] = has_rows ? cx.s_best[tid] : 0x7fffffff;
  }
  csync();
  if (tid == 0) {
    const unsigned prev = atom_release_add(P.sync + kSyncArgmax, 1u);
    *cx.s_flag = prev == static_cast<unsigned>(nct - 1);
  }
  csync();
  if (!*cx.s_flag) return;
  __threadfence();
  for (int m = warp; m < M; m += kCW) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    // every partial of this lane loaded before any is compared (one L2 round
    // trip); the order is total, so the comparison order does not matter
    constexpr int kPerLane = 8;  // up to 256 CTAs in registers
    float vv[kPerLane];
    int iv[kPerLane];
#pragma unroll
    for (int j = 0; j < kPerLane; ++j) {
      const int q = lane + 32 * j;
      vv[j] = q < nct ? __ldcg(P.am_val + static_cast<size_t>(q) * M + m) : -INFINITY;
      iv[j] = q < nct ? __ldcg(P.am_idx + static_cast<size_t>(q) * M + m) : 0x7fffffff;
    }
#pragma unroll
    for (int j = 0; j < kPerLane; ++j)
      if (am_better(vv[j], iv[j], bv, bi)) {
        bv = vv[j];
        bi = iv[j];
      }
    for (int q = lane + 32 * kPerLane; q < nct; q += 32) {
      const float v = __ldcg(P.am_val + static_cast<size_t>(q) * M + m);
      const int ix = __ldcg(P.am_idx + static_cast<size_t>(q) * M + m);
      if (am_better(v, ix, bv, bi)) {
        bv = v;
        bi = ix;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (am_better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) cx.s_best[m] = bi;
  }
  csync();
  // same feedback as gemv_argmax_finish (gemv_epi.cuh)
  if (P.mode == SB_MODE_VERIFY) {
    if (tid < M && P.out_ids) P.out_ids[tid] = cx.s_best[tid];
    if (tid == 0) {
      int j = 0;
      while (j < M - 1 && static_cast<int64_t>(cx.s_best[j]) == P.ids[j + 1]) ++j;
      P.ctrl[SB_CTRL_ACCEPT] = j;
    }
  } else {
    for (int b = tid; b < M; b += kCW * 32) {
      const int64_t tok = cx.s_best[b];
      int64_t out = tok, next = tok;
      if (P.finished) {
        if (P.finished[b]) {
          out = P.pad_id;
          next = P.pad_id;
        } else if (tok == P.eos_id) {
          P.finished[b] = 1;
          next = P.pad_id;
        }
      }
      if (P.out_ids) P.out_ids[static_cast<size_t>(P.step) * P.batch + b] = out;
      P.ids[b] = next;
    }
    if (tid == 0 && P.mode == SB_MODE_DECODE) P.ctrl[SB_CTRL_SLOT] += 1;
  }
  // every CTA has passed its last wait: reset the counters for the next launch
  // and advance the sequence number (new epochs for the handed-over words)
  const unsigned seq = P.sync[kSyncSeq];
  csync();
  for (int i = tid; i < kSyncWords; i += kCW * 32) P.sync[i] = i == kSyncSeq ? seq + 1u : 0u;
}

template <int FMT, int KH, int KI>
__global__ void __launch_bounds__(kThreads, 1) k_step(const __grid_constant__ StepParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x;
  const int R = (P.n_q / P.n_kv) * P.m_per;
  const StepLayout SL = step_layout(P.ring_bytes, P.M, R, P.rounds_per_batch, P.act_bytes, P.rc_rows);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL.bars);
  uint64_t* empty = full + kNBar;
  int32_t* err = P.ctrl + SB_CTRL_ERR;
  const int slot = P.ctrl[SB_CTRL_SLOT], pad_len = P.ctrl[SB_CTRL_PADLEN];
  if (tid == 0) {
    for (int i = 0; i < kNBar; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kCW);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (tid >= kCW * 32) {  // ---- producer warp: the whole step's weight stream
    if (tid != kCW * 32) return;
    Prod pr;
    pr.ring = smem;
    pr.ring_bytes = static_cast<uint32_t>(P.ring_bytes);
    pr.full = full;
    pr.empty = empty;
    pr.endv = reinterpret_cast<uint32_t*>(smem + SL.endv);
    pr.err = err;
    pr.rp.phys = 0;
    pr.rp.voff = 0;
    pr.rp.ei = 0;
    pr.rel_end = 0;
    pr.rel = 0;
    pr.txv = pr.endv + kNBar;
    pr.landed = 0;
    pr.inflight = 0;
    pr.cap = static_cast<uint32_t>(P.inflight_cap);
    pr.stop = false;
    const AttnUnit au = attn_unit(P, slot, pad_len);
    for (int l = 0; l < P.n_layers; ++l) {
      const StepLayer& L = P.layers[l];
      produce_vec(pr, L.in_norm, P.hidden);
      produce<FMT, KH>(pr, L.w[0], L.s[0], P.n_tiles[0]);
      if (au.active) produce_kv(pr, P, au, L, slot);
      produce<FMT, KH>(pr, L.w[1], L.s[1], P.n_tiles[1]);
      produce_vec(pr, L.post_norm, P.hidden);
      produce<FMT, KH>(pr, L.w[2], L.s[2], P.n_tiles[2]);
      produce<FMT, KI>(pr, L.w[3], L.s[3], P.n_tiles[3]);
    }
    produce_vec(pr, P.final_norm, P.hidden);
    produce<FMT, KH>(pr, P.lm_w, P.lm_s, P.n_tiles[4]);
    // do not leave while copies into this CTA's shared memory are in flight
    // (bounded, also after a failed wait): entries [landed, ei) may be in flight, and
    // only the last kNBar of them still own their barrier phase
    const int armed = pr.rp.ei;
    for (int j = max(pr.landed, armed - kNBar); j < armed; ++j)
      if (!mbar_drain(full + j % kNBar, static_cast<uint32_t>((j / kNBar) & 1), err)) break;
    return;
  }

  Cx cx;
  cx.ring = smem;
  cx.ring_bytes = static_cast<uint32_t>(P.ring_bytes);
  cx.full = full;
  cx.empty = empty;
  cx.red = reinterpret_cast<float*>(smem + SL.red);
  cx.tot = reinterpret_cast<float*>(smem + SL.tot);
  cx.s_ss = reinterpret_cast<float*>(smem + SL.ss);
  cx.s_shift = reinterpret_cast<int*>(smem + SL.shift);
  cx.xs = reinterpret_cast<uint16_t*>(smem + SL.xs);
  cx.s_best = reinterpret_cast<int*>(smem + SL.best);
  cx.s_bval = reinterpret_cast<float*>(smem + SL.bval);
  cx.s_flag = reinterpret_cast<int*>(smem + SL.flag);
  cx.sp = reinterpret_cast<GemvParams*>(smem + SL.sp);
  cx.aq = reinterpret_cast<uint32_t*>(smem + SL.aq);
  cx.asc = reinterpret_cast<float*>(smem + SL.asc);
  cx.err = err;
  cx.tid = tid;
  cx.warp = tid >> 5;
  cx.lane = tid & 31;
  cx.M = P.M;
  cx.nb = P.rounds_per_batch;
  cx.rp.phys = 0;
  cx.rp.voff = 0;
  cx.rp.ei = 0;
  cx.nbar = 0;
  cx.slot = slot;
  cx.pad_len = pad_len;
  uint16_t* rope = reinterpret_cast<uint16_t*>(smem + SL.rope);
  uint16_t* rc = reinterpret_cast<uint16_t*>(smem + SL.rc);
  int rt0, rnt;
  tile_range(P.n_tiles[1], rt0, rnt);  // o and down rows of this CTA (the residual rows it updates)
  const int rc_row0 = rt0 * 16, rc_n = min(rnt * 16, P.hidden - rc_row0);
  if (tid == 0) memset(cx.sp, 0, sizeof(GemvParams));
  // RoPE rows at each token's position (the q/k/v epilogue's cos / sin) and
  // this CTA's residual rows: the layer-0 residual is the scaled embedding
  for (int i = tid; i < P.M * 64; i += kCW * 32) {
    const int m = i >> 6, j = i & 63;
    const int b = m / P.m_per, mi = m % P.m_per;
    int pos = slot + mi - (P.rope_off ? P.rope_off[b] : 0);
    pos = pos < 0 ? 0 : (pos >= P.rope_max ? P.rope_max - 1 : pos);
    rope[m * 128 + j] = P.cos_tab[pos * 64 + j];
    rope[m * 128 + 64 + j] = P.sin_tab[pos * 64 + j];
  }
  for (int i = tid; i < P.M * rc_n; i += kCW * 32) {
    const int m = i / rc_n, r = i % rc_n;
    int64_t id = P.ids[m];
    id = id < 0 ? 0 : (id >= P.vocab ? P.vocab - 1 : id);
    rc[m * P.rc_rows + r] =
        f_to_bf16_bits(bf(u16_to_f(P.embed[static_cast<size_t>(id) * P.hidden + rc_row0 + r]) * P.emb_mult));
  }

  // Phases hand their outputs over as epoch-tagged words: a phase polls its
  // input words instead of waiting at a grid barrier.
  const unsigned seq = P.sync[kSyncSeq];
  for (int l = 0; l < P.n_layers; ++l) {
    // q/k/v: RMSNorm (layer 0: embedding x12) -> RoPE, cache rows at ctrl[SLOT] + token
    if (tid == 0) set_epi(P, cx, 0, l, rope, rc);
    gemv_phase<FMT, KH, EPI_QKV>(P, cx, P.n_tiles[0], l == 0 ? PRO_EMBED : PRO_RMSNORM, P.ll_h,
                                 l == 0 ? 0u : ll_epoch(seq, l - 1, LL_H_DOWN), ll_epoch(seq, l, LL_QKV));
    attn_phase(P, cx, l, ll_epoch(seq, l, LL_QKV), ll_epoch(seq, l, LL_ATTN));
    csync();
    // o -> residual
    if (tid == 0) set_epi(P, cx, 1, l, rope, rc);
    gemv_phase<FMT, KH, EPI_RESID>(P, cx, P.n_tiles[1], PRO_NONE, P.ll_attn, ll_epoch(seq, l, LL_ATTN),
                                   ll_epoch(seq, l, LL_H_O));
    csync();
    // gate/up: RMSNorm -> SiLU(gate) * up
    if (tid == 0) set_epi(P, cx, 2, l, rope, rc);
    gemv_phase<FMT, KH, EPI_SWIGLU>(P, cx, P.n_tiles[2], PRO_RMSNORM, P.ll_h, ll_epoch(seq, l, LL_H_O),
                                    ll_epoch(seq, l, LL_ACT));
    csync();
    // down -> residual
    if (tid == 0) set_epi(P, cx, 3, l, rope, rc);
    gemv_phase<FMT, KI, EPI_RESID>(P, cx, P.n_tiles[3], PRO_NONE, P.ll_act, ll_epoch(seq, l, LL_ACT),
                                   ll_epoch(seq, l, LL_H_DOWN));
    csync();
  }
  // final norm -> lm_head -> argmax
  if (tid == 0) set_epi(P, cx, 4, 0, rope, rc);
  gemv_phase<FMT, KH, EPI_ARGMAX>(P, cx, P.n_tiles[4], PRO_RMSNORM, P.ll_h, ll_epoch(seq, P.n_layers - 1, LL_H_DOWN),
                                  0u);
  int t0, nt;
  tile_range(P.n_tiles[4], t0, nt);
  lm_finish(P, cx, nt > 0);
}

}  // namespace

// ---- host side ------------------------------------------------------------------
static const size_t kStepSmemMax = 227 * 1024;

struct DevInfo {
  int sms = 0, coop = 0;
};
static DevInfo dev_info() {
  static DevInfo info[16];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 16) return DevInfo();
  if (info[dev].sms == 0) {
    cudaDeviceGetAttribute(&info[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&info[dev].coop, cudaDevAttrCooperativeLaunch, dev);
  }
  return info[dev];
}

// Weight bytes one CTA keeps in flight at most (>= one 40 KiB entry).  Deeper
// queues do not raise the stream's bandwidth (the step consumes far below it
// between grid barriers) but add their queueing delay to the step's
// latency-critical activation reads.
static int inflight_cap() { return 48 * 1024; }

// (hidden, inter) shapes with a compiled kernel
static bool dims_supported(int hidden, int inter) {
  return (hidden == 2048 && inter == 8192) || (hidden == 512 && inter == 1024);
}

static int split_for(int max_len) { return (max_len + kStepKeys - 1) / kStepKeys; }

// words of the handed-over activations per token
static size_t ll_words(const SbModel* md) {
  return static_cast<size_t>(md->hidden) / 2 + md->n_q * 64 * 2 + md->n_kv * 128 + md->inter / 2;
}

size_t step_ws_bytes(const SbModel* md, int tokens) {
  if (tokens < 1 || tokens > 8) return 0;
  const size_t rows = static_cast<size_t>(tokens) * md->n_q;  // batch * n_kv * R
  const size_t stats = rows * kStepMaxSplit * sizeof(float2);
  const size_t part = rows * kStepMaxSplit * 128 * 4;
  const size_t am = static_cast<size_t>(256) * tokens * 8;
  return kSyncWords * 4 + stats + part + am + static_cast<size_t>(tokens) * ll_words(md) * 8;
}

bool step_plan(const SbModel* md, const SbState* st, StepPlan& pl, const char** why) {
  auto no = [&](const char* w) {
    if (why) *why = w;
    return false;
  };
  const int T = st->batch * st->m;
  if (T < 1 || T > 8) return no("more than 8 token rows");
  const DevInfo di = dev_info();
  if (!di.coop || di.sms < 1 || di.sms > 256) return no("no cooperative launch");
  if (!md->layers || md->n_layers < 1 || md->n_layers > kStepMaxLayers) return no("layer count");
  if (md->head_dim != 128 || md->n_q * 128 != md->hidden || md->n_q % md->n_kv) return no("head layout");
  if (!dims_supported(md->hidden, md->inter)) return no("hidden / intermediate size");
  const int fmt = md->lm_head.fmt;
  auto same = [&](const SbLinear& l, int n, int k) {
    return l.w && l.fmt == fmt && l.n == n && l.k == k && l.n_pad % 16 == 0 && l.n_pad >= n &&
           (fmt == SB_FMT_BF16 || l.scale);
  };
  if (!same(md->lm_head, md->vocab, md->hidden)) return no("lm_head");
  for (int i = 0; i < md->n_layers; ++i) {
    const SbLayer& L = md->layers[i];
    if (!same(L.qkv, (md->n_q + 2 * md->n_kv) * 128, md->hidden) || !same(L.o, md->hidden, md->hidden) ||
        !same(L.gate_up, 2 * md->inter, md->hidden) || !same(L.down, md->hidden, md->inter) || !L.k_cache ||
        !L.v_cache || !L.in_norm || !L.post_norm)
      return no("layer weights (one format for every projection)");
  }
  const int R = (md->n_q / md->n_kv) * st->m;
  if (R > kStepMaxRows) return no("query rows per KV head");
  const int ns = split_for(md->max_len);
  if (ns > kStepMaxSplit || st->batch * md->n_kv * ns > di.sms) return no("attention splits");
  if (st->batch * md->n_kv > 1024) return no("streams x KV heads");
  pl.fmt = fmt;
  pl.n_split = ns;
  pl.rows = R;
  pl.rounds_per_batch = 16 / T;
  pl.grid = di.sms;
  const size_t ah = step_act_bytes(fmt, md->hidden, T), ai = step_act_bytes(fmt, md->inter, T);
  pl.act_bytes = ah > ai ? ah : ai;
  const int hidden_tiles = md->layers[0].o.n_pad / 16;
  pl.rc_rows = (hidden_tiles + pl.grid - 1) / pl.grid * 16;
  const size_t fixed = step_layout(0, T, R, pl.rounds_per_batch, pl.act_bytes, pl.rc_rows).total;
  if (fixed + 48 * 1024 > kStepSmemMax) return no("shared memory");
  pl.ring_bytes = static_cast<int>((kStepSmemMax - fixed) / 128 * 128);
  pl.smem = step_layout(pl.ring_bytes, T, R, pl.rounds_per_batch, pl.act_bytes, pl.rc_rows).total;
  if (pl.smem > kStepSmemMax) return no("shared memory");
  return true;
}

template <int FMT, int KH, int KI>
static int launch_t(const StepParams& P, const StepPlan& pl, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  static unsigned configured = 0;
  if (!(configured & (1u << dev))) {
    cudaError_t e = cudaFuncSetAttribute(k_step<FMT, KH, KI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kStepSmemMax));
    if (e != cudaSuccess) return e;
    configured |= 1u << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&cfg, k_step<FMT, KH, KI>, P);
}

template <int FMT>
static int launch_f(const StepParams& P, const StepPlan& pl, cudaStream_t s) {
  if (P.hidden == 2048) return launch_t<FMT, 2048, 8192>(P, pl, s);
  return launch_t<FMT, 512, 1024>(P, pl, s);
}

int step_launch(const SbModel* md, const SbState* st, int step, void* ws, const StepPlan& pl, cudaStream_t s) {
  StepParams P;
  memset(&P, 0, sizeof(P));
  P.n_layers = md->n_layers;
  P.hidden = md->hidden;
  P.inter = md->inter;
  P.n_q = md->n_q;
  P.n_kv = md->n_kv;
  P.vocab = md->vocab;
  P.max_len = md->max_len;
  P.rope_max = md->rope_max_pos;
  const SbLayer& L0 = md->layers[0];
  const SbLinear* mats[5] = {&L0.qkv, &L0.o, &L0.gate_up, &L0.down, &md->lm_head};
  for (int i = 0; i < 5; ++i) {
    P.n_tiles[i] = mats[i]->n_pad / 16;
    P.n_rows[i] = mats[i]->n;
  }
  P.eps = md->eps;
  P.attn_mult = md->attn_mult;
  P.emb_mult = md->emb_mult;
  P.res_mult = md->res_mult;
  P.logits_mult = md->logits_mult;
  P.embed = md->embed;
  P.final_norm = md->final_norm;
  P.cos_tab = md->rope_cos;
  P.sin_tab = md->rope_sin;
  P.lm_w = static_cast<const uint8_t*>(md->lm_head.w);
  P.lm_s = static_cast<const uint8_t*>(md->lm_head.scale);
  P.lm_g = md->lm_head.global_scale;
  P.batch = st->batch;
  P.m_per = st->m;
  P.M = st->batch * st->m;
  P.mode = st->mode;
  P.step = step;
  P.ids = st->ids;
  P.ctrl = st->ctrl;
  P.prompt_len = st->prompt_len;
  P.rope_off = st->rope_off;
  P.finished = st->finished;
  P.out_ids = st->out_ids;
  P.resid = st->hidden;
  P.q = st->q;
  P.attn = st->attn;
  P.act = st->act;
  P.logits = st->logits;
  P.eos_id = st->eos_id;
  P.pad_id = st->pad_id;
  const size_t rows = static_cast<size_t>(P.M) * md->n_q;
  char* b = static_cast<char*>(ws);
  P.sync = reinterpret_cast<unsigned*>(b);
  P.attn_stats = reinterpret_cast<float2*>(b + kSyncWords * 4);
  P.attn_part = reinterpret_cast<float*>(b + kSyncWords * 4 + rows * kStepMaxSplit * sizeof(float2));
  P.am_val = reinterpret_cast<float*>(b + kSyncWords * 4 + rows * kStepMaxSplit * (sizeof(float2) + 512));
  P.am_idx = reinterpret_cast<int*>(reinterpret_cast<char*>(P.am_val) + static_cast<size_t>(256) * P.M * 4);
  unsigned long long* ll = reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(P.am_idx) +
                                                                 static_cast<size_t>(256) * P.M * 4);
  P.ll_h = ll;
  P.ll_q = P.ll_h + static_cast<size_t>(P.M) * md->hidden / 2;
  P.ll_kv = P.ll_q + static_cast<size_t>(P.M) * md->n_q * 64;
  P.ll_attn = P.ll_kv + static_cast<size_t>(P.M) * md->n_kv * 128;
  P.ll_act = P.ll_attn + static_cast<size_t>(P.M) * md->n_q * 64;
  P.n_split = pl.n_split;
  P.ring_bytes = pl.ring_bytes;
  P.rounds_per_batch = pl.rounds_per_batch;
  P.act_bytes = static_cast<int>(pl.act_bytes);
  P.inflight_cap = inflight_cap();
  P.rc_rows = pl.rc_rows;
  for (int l = 0; l < md->n_layers; ++l) {
    const SbLayer& L = md->layers[l];
    StepLayer& D = P.layers[l];
    D.in_norm = L.in_norm;
    D.post_norm = L.post_norm;
    const SbLinear* lin[4] = {&L.qkv, &L.o, &L.gate_up, &L.down};
    for (int i = 0; i < 4; ++i) {
      D.w[i] = static_cast<const uint8_t*>(lin[i]->w);
      D.s[i] = static_cast<const uint8_t*>(lin[i]->scale);
      D.g[i] = lin[i]->global_scale;
    }
    D.k_cache = L.k_cache;
    D.v_cache = L.v_cache;
  }
  switch (pl.fmt) {
    case SB_FMT_BF16: return launch_f<SB_FMT_BF16>(P, pl, s);
    case SB_FMT_FP8: return launch_f<SB_FMT_FP8>(P, pl, s);
    case SB_FMT_INT8: return launch_f<SB_FMT_INT8>(P, pl, s);
    case SB_FMT_NVFP4: return launch_f<SB_FMT_NVFP4>(P, pl, s);
  }
  return SB_ERR_ARG;
}

}  // namespace sb
