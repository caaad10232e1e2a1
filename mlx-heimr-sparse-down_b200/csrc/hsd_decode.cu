// Sparse MoE down projection for decode on the neuron-major layout (hsd/decode.py).
//
//   y[b, o] = sum_k gains[b,k] * sum_{i : h[b,k,i] != 0} h[b,k,i] * W_{sel[b,k]}[o, i]
//           + gains[b,topk]   * sum_{i : hs[b,i] != 0}  hs[b,i]  * Ws[o, i]
//   W[o, i] = s[i/64, o] * q[i, o] + b[i/64, o]           (affine 4-bit, group 64)
//
// Work split (one token = one row b of h):
//   The token's 64-neuron groups are listed slot by slot (topk routed experts, then the
//   shared expert): GT = topk*F/64 + FS/64 groups (232 at the reference shapes); they are
//   the contiguous 64-column blocks of h's row. The D outputs are cut into chunks of C
//   outputs (C/2 contiguous bytes of every neuron row). A thread-block CLUSTER of 8 CTAs
//   owns one (token, chunk); CTA `rank` owns groups [rank*GT/8, (rank+1)*GT/8) -- at the
//   reference shapes one routed expert or one half of the shared expert (29 groups). The 8
//   partial outputs are summed through distributed shared memory in a fixed rank order:
//   deterministic, with no scratch memory, atomics or second kernel.
//
// Per CTA and batch of up to 32 groups:
//   1. one 16-byte load per thread brings the batch's h columns (and each group's expert
//      id and gain) into shared memory;
//   2. each warp builds its groups' live masks with two ballots and, for a live group,
//      starts the copies of the group's scale and bias chunks (C*2 bytes each) as 16-byte
//      cp.async pieces, one per lane;
//   3. every warp scans the live counts, cuts the live rows into sub-batches of whole groups
//      of at most SBR rows, and compacts its groups' live rows into an ascending list
//      (ballot prefix popcounts); each lane holding a live row of one of the first `slots`
//      sub-batches starts the copy of that row's C/2-byte chunk into the sub-batch's slot of
//      the shared-memory ring as one TMA bulk copy. The TMA unit takes one bulk copy about
//      every 16 cycles, which makes the issue of the ~200 row copies per CTA the longest
//      phase of a token's chain; the scale/bias pieces of step 2 go over the load/store
//      path, beside it, instead of adding ~60 bulk copies to that queue. A slot's copies
//      complete on the slot's mbarrier: one arrival carries the sub-batch's TMA bytes, and
//      every thread adds one arrival that fires when its own cp.async pieces have landed;
//   4. per sub-batch, as its slot's mbarrier completes: thread (word wp, group lane gl)
//      walks the live rows of its groups gl, gl+NGL, ... of the sub-batch in shared memory,
//      accumulating acc'[n] = sum h * (1 + q_n/16) and hsum = sum h in fp32, and folds each
//      group in as out[n] += g * (16*s[n]*(acc'[n] - hsum) + b[n]*hsum) -- the reference's
//      affine algebra (s * sum(h q) + b * sum(h)); 1 + q/16 is built exactly from the
//      nibble with bit operations, sparing an integer-to-float conversion per weight. The
//      computation of a sub-batch overlaps the landing of the later ones; a slot freed is
//      refilled with the sub-batch `slots` places later;
//   5. the NGL group lanes are reduced in shared memory in a fixed order;
//   6. each CTA pushes the 8 slices of its partial chunk to their owner CTAs with st.async
//      (completing on the owner's mbarrier), and each owner sums its slice's 8 partials in
//      rank order: one cluster handshake (at the start) instead of two cluster barriers.
// A lane's groups are folded in ascending order whatever the sub-batch cut, and a group's
// rows always form one sub-batch, so the result depends neither on the ring's size nor on
// the other groups' live counts: the dense form (every row live) and the sparse form give
// the same bits, and so do every stage size chosen per batch size below.
// Weights are streamed with an L2 evict-first policy (they are not reused by the step).
// The launch uses programmatic dependent launch: the kernel releases its dependents at
// once and waits (griddepcontrol.wait) for the previous kernel before its first read, so
// back-to-back layers overlap launch latency with the previous layer's tail. Every
// mbarrier wait is bounded (2 s of %globaltimer); running out sets HSD_ERR_TIMEOUT in the
// status word, waits once more (bounded) for the copies in flight and finishes.
#include <cooperative_groups.h>
#include <cstdlib>

#include "hsd_common.cuh"

namespace cg = cooperative_groups;

HSD_DEFINE_STATUS(decode)

namespace {

constexpr int kCluster = 8;    // CTAs per (token, chunk)
constexpr int kGB = 32;        // groups per batch
constexpr int kGS = 64;        // quantisation group size
constexpr int kMaxSlots = 8;   // sub-batch slots (mbarriers) of the staging ring

template <int C>
struct DecodeCfg {
  static constexpr int NWC = C / 8;                    // words of one row in a chunk
  static constexpr int THREADS = 512;                  // 16 full warps (ballots use full masks)
  static constexpr int WARPS = THREADS / 32;
  static constexpr int NGL = WARPS;                    // group lanes: one warp each, a lane per word
  static_assert(NWC <= 32, "a chunk row must fit one warp");
  static constexpr int MAX_RB = 1024;                  // largest staging ring, in rows
  static constexpr int MIN_RB = NGL * 8;               // the group-lane partials reuse the ring
};

struct DecodeParams {
  const void* h;
  const int32_t* sel;
  const float* gains;
  const uint32_t* pw;
  const uint16_t* ps;
  const uint16_t* pb;
  const uint32_t* spw;
  const uint16_t* sps;
  const uint16_t* spb;
  const void* resid;
  void* y;
  int B, D, F, FS, topk, E, loadsc;
  int all_rows;   // 1: every row of the selected experts is live (the dense form)
  int NR;    // columns of h: topk*F + FS
  int GT;    // groups per token
  int NW;    // words per neuron row: D/8
  int SBR;   // rows per ring slot = the sub-batch limit (>= 64: a group's rows fit one slot)
  int nring; // slots of the staging ring (ring rows = SBR * nring), 1..kMaxSlots
};

// The staging ring (SBR*nring rows of NWC words, also the group-lane partials) follows this
// struct in dynamic shared memory, at a 128-byte boundary.
template <int C>
struct DecodeSmem {
  using Cfg = DecodeCfg<C>;
  uint16_t meta_s[kGB * C];                     // staged scale chunks (16-bit)
  uint16_t meta_b[kGB * C];                     // staged bias chunks
  float hs[kGB * kGS];                          // the batch's h values (fp32)
  float hrow[kGB * kGS];                        // h of each compacted live row
  uint16_t rows[kGB * kGS];                     // compacted live rows: (group in batch) << 6 | neuron
  unsigned long long gmask[kGB];
  unsigned long long bars[kMaxSlots];           // completion of each slot's bulk copies
  unsigned long long rbar;                      // arrival of the 8 partial slices (st.async)
  int gcnt[kGB], goff[kGB + 1];
  int sbeg[kGB + 1];                            // sub-batch starts (rows); sbeg[nsb] = nrows
  int gsrc[kGB];                                // expert id, -1 = shared expert, -2 = invalid
  int gloc[kGB];                                // the group's index inside its expert
  float ggain[kGB];
  float part[C];                                // this CTA's partial output chunk
  float recv[C];                                // [rank][C/8]: the slices pushed to this CTA
};

template <int C>
constexpr size_t ring_offset() {
  return (sizeof(DecodeSmem<C>) + 127) / 128 * 128;
}

// Live mask of 64 h values (two per lane) with two ballots.
__device__ __forceinline__ unsigned long long ballot64(bool nz0, bool nz1) {
  const unsigned lo = __ballot_sync(0xffffffffu, nz0);
  const unsigned hi = __ballot_sync(0xffffffffu, nz1);
  return (static_cast<unsigned long long>(hi) << 32) | lo;
}

// Index of this lane's entry (j = lane or lane + 32) among the live entries of mask.
__device__ __forceinline__ int live_prefix(unsigned long long mask, int j) {
  const unsigned long long below = (j == 0) ? 0ull : (mask & ((1ull << j) - 1ull));
  return __popcll(below);
}

// 1 + q/16 for the nibble of q at bit offset 4n, exact: q lands in mantissa bits 19..22.
template <int N>
__device__ __forceinline__ float nib_unit(uint32_t q) {
  constexpr int sh = 19 - 4 * N;
  const uint32_t m = (sh >= 0) ? (q << (sh >= 0 ? sh : 0)) : (q >> (sh < 0 ? -sh : 0));
  return __uint_as_float((m & 0x00780000u) | 0x3F800000u);
}

// (x, y) = (fma(h, u, x), fma(h, v, y)), each rounded to nearest as fmaf does: one packed
// fp32 FMA (fma.rn.f32x2, sm_100) in place of two, the same bits
__device__ __forceinline__ void ffma2(float& x, float& y, float h, float u, float v) {
  asm("{\n .reg .b64 a, b, c;\n mov.b64 a, {%2, %2};\n mov.b64 b, {%3, %4};\n mov.b64 c, {%0, %1};\n"
      " fma.rn.f32x2 c, a, b, c;\n mov.b64 {%0, %1}, c;\n}"
      : "+f"(x), "+f"(y) : "f"(h), "f"(u), "f"(v));
}

template <typename HT>
__device__ __forceinline__ float load_h(const void* h, int64_t idx) {
  return hsd::to_f32<HT>(reinterpret_cast<const HT*>(h)[idx]);
}

// ---- mbarrier / bulk-copy helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}"
               ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait for the phase with `parity`: false after ~2 s.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > 2000000000ull) return false;
  return true;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// One TMA bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}

// 16 bytes global -> this CTA's shared memory on the load/store path (cp.async, L2 hint),
// beside the TMA unit: the two paths issue in parallel.
__device__ __forceinline__ void cp16(void* dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;"
               ::"r"(smem_u32(dst)), "l"(src), "l"(pol) : "memory");
}
// One arrival on `bar` once every cp.async this thread issued before it has landed (the
// barrier's expected count includes one such arrival per thread).
__device__ __forceinline__ void cp_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// ---- distributed shared memory helpers
// The address of this CTA's shared-memory location `a` in cluster CTA `r`.
__device__ __forceinline__ uint32_t mapa_u32(uint32_t a, uint32_t r) {
  uint32_t o;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(o) : "r"(a), "r"(r));
  return o;
}
// A 4-byte store into another cluster CTA's shared memory, counted on that CTA's mbarrier.
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];"
               ::"r"(addr), "f"(v), "r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait (cluster-scope acquire) for the phase with `parity`: false after ~2 s.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait_cluster(bar, parity))
    if (global_ns() - t0 > 2000000000ull) return false;
  return true;
}

template <typename HT, typename ST, typename YT, int C>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(DecodeCfg<C>::THREADS)
    sparse_down_decode_kernel(const DecodeParams p) {
  using Cfg = DecodeCfg<C>;
  constexpr int NWC = Cfg::NWC, NGL = Cfg::NGL, THREADS = Cfg::THREADS, WARPS = Cfg::WARPS;
  constexpr int HPV = 16 / sizeof(HT);           // h values per 16-byte load
  extern __shared__ __align__(128) unsigned char smem_raw[];
  DecodeSmem<C>& S = *reinterpret_cast<DecodeSmem<C>*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rank = static_cast<int>(cluster.block_rank());
  const int ch = blockIdx.x / kCluster;
  const int b = blockIdx.y;
  const int w0 = ch * NWC;                        // first word of this chunk
  const int nwc = min(NWC, p.NW - w0);            // words of this chunk (tail chunk may be short)
  const int GF = p.F / kGS;
  const int g_lo = static_cast<int>((static_cast<long long>(rank) * p.GT) / kCluster);
  const int g_hi = static_cast<int>((static_cast<long long>(rank + 1) * p.GT) / kCluster);
  // A group lane is a warp and its lane wp owns word wp of the chunk: the lanes of a warp
  // walk the same rows, so the row loop never diverges (C < 256 leaves lanes idle).
  const int wp = lane;                            // word of the chunk this thread owns
  const int gl = warp;                            // group lane
  const bool lane_used = wp < NWC;
  const bool active = wp < nwc;
  uint32_t* ring = reinterpret_cast<uint32_t*>(smem_raw + ring_offset<C>());
  const int SBR = p.SBR, nring = p.nring;
  const uint32_t bar0 = smem_u32(&S.bars[0]);     // slot k's mbarrier: bar0 + 8*k
  const uint32_t rbar = smem_u32(&S.rbar);
  const uint32_t row_bytes = static_cast<uint32_t>(nwc) * 4;
  constexpr int per = C / kCluster;               // outputs of the chunk each CTA finishes
  uint32_t phases = 0;                            // bit k: the parity slot k waits for next
  const uint64_t pol = evict_first_policy();

  if (tid == 0) {
    // a slot's phase: the arrival carrying its TMA bytes + one cp.async arrival per thread
    for (int k = 0; k < kMaxSlots; ++k) mbar_init(bar0 + 8u * k, 1 + THREADS);
    mbar_init(rbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // the 8 slices of C/8 partials that the cluster's CTAs push here complete this phase
    mbar_arrive_expect_tx(rbar, static_cast<uint32_t>(sizeof(float) * C));
  }
  __syncthreads();
  // the handshake that makes every CTA's mbarriers visible before any push (waited in 6.)
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  // Programmatic dependent launch: let the next kernel in the stream start its launch
  // now, and wait for the previous one (which produces h / sel / gains) before reading.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  float out[8];
#pragma unroll
  for (int n = 0; n < 8; ++n) out[n] = 0.f;

  for (int gb0 = g_lo; gb0 < g_hi; gb0 += kGB) {
    const int ng = min(kGB, g_hi - gb0);
    // the previous batch's shared-memory reads come before this batch's bulk copies
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // ---- 1. h columns [64*gb0, 64*(gb0+ng)) of row b, the groups' expert ids and gains
    {
      const HT* hrow = reinterpret_cast<const HT*>(p.h) + static_cast<int64_t>(b) * p.NR +
                       static_cast<int64_t>(gb0) * kGS;
      for (int v = tid; v < ng * kGS / HPV; v += THREADS) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(hrow) + v);
        const HT* e = reinterpret_cast<const HT*>(&raw);
        float f[HPV];
#pragma unroll
        for (int i = 0; i < HPV; ++i) f[i] = hsd::to_f32<HT>(e[i]);
#pragma unroll
        for (int i = 0; i < HPV; i += 4)
          *reinterpret_cast<float4*>(&S.hs[v * HPV + i]) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
      }
      if (tid < ng) {
        const int G = gb0 + tid;
        int slot, loc, src;
        if (G < p.topk * GF) {
          slot = G / GF;
          loc = G - slot * GF;
          src = __ldg(p.sel + static_cast<int64_t>(b) * p.topk + slot);
          if (src < 0 || src >= p.E) {
            hsd_flag_decode(HSD_ERR_INDEX);
            src = -2;
          }
        } else {
          slot = p.topk;
          loc = G - p.topk * GF;
          src = -1;
        }
        S.gsrc[tid] = src;
        S.gloc[tid] = loc;
        S.ggain[tid] = __ldg(p.gains + static_cast<int64_t>(b) * (p.topk + 1) + slot);
      }
    }
    __syncthreads();
    // ---- 2. live masks (one warp per group)
    for (int gi = warp; gi < ng; gi += WARPS) {
      const bool valid = S.gsrc[gi] != -2;
      const float v0 = valid ? S.hs[gi * kGS + lane] : 0.f;
      const float v1 = valid ? S.hs[gi * kGS + 32 + lane] : 0.f;
      const unsigned long long m = p.all_rows ? ballot64(valid, valid) : ballot64(v0 != 0.f, v1 != 0.f);
      if (lane == 0) {
        S.gmask[gi] = m;
        S.gcnt[gi] = __popcll(m);
      }
      if (m != 0ull && p.loadsc && lane < nwc) {   // a live group's scale and bias chunks: 16 bytes a lane
        const int src = S.gsrc[gi];
        const int64_t grow = (src >= 0) ? static_cast<int64_t>(src) * GF + S.gloc[gi] : S.gloc[gi];
        const int64_t go = grow * p.D + static_cast<int64_t>(w0) * 8 + lane * 8;
        cp16(S.meta_s + gi * C + lane * 8, ((src >= 0) ? p.ps : p.sps) + go, pol);   // complete on slot 0
        cp16(S.meta_b + gi * C + lane * 8, ((src >= 0) ? p.pb : p.spb) + go, pol);
      }
    }
    __syncthreads();
    // ---- 3. the counts' exclusive scan and the sub-batch cut (every warp, redundantly),
    //         the compaction and the row copies of the first nring sub-batches
    int nsb = 0;
    {
      const int c = (lane < ng) ? S.gcnt[lane] : 0;
      int x = c;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
      }
      const int goff_lane = x - c;                 // group `lane`'s rows: [goff_lane, x)
      const int nrows = __shfl_sync(0xffffffffu, x, 31);
      // greedy cut into sub-batches of whole groups of at most SBR rows (a group never
      // straddles two, so it is always folded in one piece: a group's sum is the same
      // sequence of fp32 operations whatever the other groups' live counts). Lane k ends
      // holding sub-batch k's first row (my_sbeg) and last row + 1 (my_send); my_sb is the
      // sub-batch of group `lane`.
      int my_sbeg = 0, my_sb = 0;
      for (int start = 0; start < nrows; ++nsb) {
        const unsigned cand = (lane < ng && x > start && x - start <= SBR) ? static_cast<unsigned>(x) : 0u;
        const int nxt = static_cast<int>(__reduce_max_sync(0xffffffffu, cand));
        if (lane == nsb) my_sbeg = start;
        if (lane < ng && goff_lane >= start && goff_lane < nxt) my_sb = nsb;
        start = nxt;
      }
      if (lane == nsb) my_sbeg = nrows;
      const int next_beg = __shfl_down_sync(0xffffffffu, my_sbeg, 1);
      const int my_send = (lane + 1 >= nsb) ? nrows : next_beg;
      if (warp == 0) {
        if (lane < ng) S.goff[lane] = goff_lane;
        if (lane == 0) S.goff[ng] = nrows;
        if (lane < nsb) S.sbeg[lane] = my_sbeg;
        if (lane == 0) S.sbeg[nsb] = nrows;
        // each in-flight sub-batch's TMA byte count (its rows), registered once with its
        // slot's arrival (copies already issued may complete first: the phase cannot end
        // before the arrivals); the cp.async scale/bias chunks complete on slot 0 through
        // the threads' cp.async arrivals
        if (lane < min(nsb, nring))
          mbar_arrive_expect_tx(bar0 + 8u * lane, static_cast<uint32_t>(my_send - my_sbeg) * row_bytes);
      }
      for (int gi = warp; gi < ng; gi += WARPS) {
        const unsigned long long m = S.gmask[gi];
        const int base = __shfl_sync(0xffffffffu, goff_lane, gi);
        const int sb = __shfl_sync(0xffffffffu, my_sb, gi);
        const int sb_first = __shfl_sync(0xffffffffu, my_sbeg, sb & 31);
        const int src = S.gsrc[gi];
        const int64_t rowbase = (src >= 0) ? (static_cast<int64_t>(src) * p.F + static_cast<int64_t>(S.gloc[gi]) * kGS)
                                           : static_cast<int64_t>(S.gloc[gi]) * kGS;
        const uint32_t* wbase = (src >= 0) ? p.pw : p.spw;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int j = lane + 32 * half;
          if ((m >> j) & 1ull) {
            const int idx = base + live_prefix(m, j);
            S.rows[idx] = static_cast<uint16_t>((gi << 6) | j);
            S.hrow[idx] = S.hs[gi * kGS + j];
            if (sb < nring) {
              uint32_t* dst = ring + static_cast<size_t>(sb * SBR + idx - sb_first) * NWC;
              const uint32_t* src = wbase + (rowbase + j) * p.NW + w0;
              bulk_g2s(dst, src, row_bytes, bar0 + 8u * sb, pol);
            }
          }
        }
      }
      // one cp.async arrival per thread on every slot in flight (the scale/bias pieces land
      // with slot 0's phase)
      for (int k = 0; k < min(nsb, nring); ++k) cp_arrive(bar0 + 8u * k);
    }
    __syncthreads();

    // ---- 4. per sub-batch, as its slot's copies land: accumulate from shared memory, then
    //         refill the slot with the sub-batch nring places later
    for (int k = 0; k < nsb; ++k) {
      const int r0 = S.sbeg[k], r1 = S.sbeg[k + 1];
      const int sk = k % nring;
      const uint32_t bk = bar0 + 8u * sk;
      const uint32_t* stage = ring + static_cast<size_t>(sk) * SBR * NWC;
      if (!mbar_wait_bounded(bk, (phases >> sk) & 1u)) {
        if (tid == 0) hsd_flag_decode(HSD_ERR_TIMEOUT);
        mbar_wait_bounded(bk, (phases >> sk) & 1u);   // once more for the copies still in flight
      }
      phases ^= 1u << sk;
      if (active) {
        for (int gi = gl; gi < ng; gi += NGL) {
          const int j0 = max(S.goff[gi], r0), j1 = min(S.goff[gi + 1], r1);
          if (j0 >= j1) continue;
          float acc[8], hsum = 0.f;
#pragma unroll
          for (int n = 0; n < 8; ++n) acc[n] = 0.f;
          for (int r = j0; r < j1; ++r) {
            const float hv = S.hrow[r];
            const uint32_t q = stage[(r - r0) * NWC + wp];
            hsum += hv;
            ffma2(acc[0], acc[1], hv, nib_unit<0>(q), nib_unit<1>(q));
            ffma2(acc[2], acc[3], hv, nib_unit<2>(q), nib_unit<3>(q));
            ffma2(acc[4], acc[5], hv, nib_unit<4>(q), nib_unit<5>(q));
            ffma2(acc[6], acc[7], hv, nib_unit<6>(q), nib_unit<7>(q));
          }
          const float g = S.ggain[gi];
          if (p.loadsc) {
            const uint4 s4 = *reinterpret_cast<const uint4*>(&S.meta_s[gi * C + wp * 8]);
            const uint4 b4 = *reinterpret_cast<const uint4*>(&S.meta_b[gi * C + wp * 8]);
            const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
            const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int n = 0; n < 8; ++n) {
              const float sc = hsd::bits16_to_f32<ST>(static_cast<uint16_t>(sw[n >> 1] >> (16 * (n & 1))));
              const float bi = hsd::bits16_to_f32<ST>(static_cast<uint16_t>(bw[n >> 1] >> (16 * (n & 1))));
              out[n] = fmaf(g, fmaf(16.f * sc, acc[n] - hsum, bi * hsum), out[n]);
            }
          } else {
#pragma unroll
            for (int n = 0; n < 8; ++n) out[n] = fmaf(g, fmaf(16.f, acc[n] - hsum, hsum), out[n]);
          }
        }
      }
      if (k + nring < nsb) {                     // refill slot sk (every thread is done with it)
        __syncthreads();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        const int q0 = S.sbeg[k + nring], qn = S.sbeg[k + nring + 1] - q0;
        if (tid == 0) mbar_arrive_expect_tx(bk, static_cast<uint32_t>(qn) * row_bytes);
        for (int r = tid; r < qn; r += THREADS) {
          const int code = S.rows[q0 + r];
          const int gi = code >> 6, j = code & 63;
          const int src = S.gsrc[gi];
          const int64_t neuron = static_cast<int64_t>(S.gloc[gi]) * kGS + j;
          const uint32_t* g = (src >= 0) ? p.pw + (static_cast<int64_t>(src) * p.F + neuron) * p.NW
                                         : p.spw + neuron * p.NW;
          uint32_t* dst = ring + (static_cast<size_t>(sk) * SBR + r) * NWC;
          bulk_g2s(dst, g + w0, row_bytes, bk, pol);
        }
        cp_arrive(bk);
      }
    }
    __syncthreads();                             // the ring, meta and hs are rewritten next
  }

  // ---- 5. reduce the group lanes (fixed order) into S.part, reusing the ring
  float* red = reinterpret_cast<float*>(ring);   // [NGL][C] fp32 (the host keeps ring >= MIN_RB rows)
  if (lane_used) {
    *reinterpret_cast<float4*>(&red[gl * C + wp * 8]) = make_float4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<float4*>(&red[gl * C + wp * 8 + 4]) = make_float4(out[4], out[5], out[6], out[7]);
  }
  __syncthreads();
  {                                              // 4 partial sums per output, then their sum
    constexpr int NP = 4, PER = (NGL + NP - 1) / NP;
    float* red2 = S.hs;                          // [NP][C] (hs is free now)
    for (int t = tid; t < NP * C; t += THREADS) {
      const int o = t % C, q = t / C;
      float a = 0.f;
#pragma unroll
      for (int l = q * PER; l < min(NGL, (q + 1) * PER); ++l) a += red[l * C + o];
      red2[q * C + o] = a;
    }
    __syncthreads();
    for (int o = tid; o < C; o += THREADS)
      S.part[o] = (red2[o] + red2[C + o]) + (red2[2 * C + o] + red2[3 * C + o]);
  }
  // ---- 6. the cluster's 8 partials: slice r of every CTA's chunk goes to CTA r (st.async,
  //         completing on CTA r's rbar), which sums the 8 slices in rank order
  __syncthreads();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");   // every rbar is initialised
  for (int o = tid; o < C; o += THREADS) {
    const int dst = o / per;
    st_async_f32(mapa_u32(smem_u32(&S.recv[rank * per + (o - dst * per)]), dst), S.part[o],
                 mapa_u32(rbar, dst));
  }
  if (!mbar_wait_cluster_bounded(rbar, 0)) {
    if (tid == 0) hsd_flag_decode(HSD_ERR_TIMEOUT);
    mbar_wait_cluster_bounded(rbar, 0);          // once more for the stores still in flight
  }
  for (int i = tid; i < per; i += THREADS) {
    const int o = rank * per + i;
    if (o < nwc * 8) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < kCluster; ++q) t += S.recv[q * per + i];
      const int64_t yi = static_cast<int64_t>(b) * p.D + static_cast<int64_t>(w0) * 8 + o;
      if (p.resid) t += hsd::to_f32<YT>(reinterpret_cast<const YT*>(p.resid)[yi]);
      reinterpret_cast<YT*>(p.y)[yi] = hsd::from_f32<YT>(t);
    }
  }
  // No CTA reads another's shared memory, and every CTA leaves only after the 8 slices
  // pushed to it have landed, so no closing cluster barrier is needed.
}

// ---- active-index sets, the same ballot compaction per (token, slot)
constexpr int kLiveThreads = 256;
constexpr int kWarps = kLiveThreads / 32;

template <typename HT>
__global__ void __launch_bounds__(kLiveThreads) live_rows_kernel(const void* h, int32_t* live,
                                                             int32_t* count, int F, int FS, int topk) {
  const int slot = blockIdx.x, b = blockIdx.y;
  const int width = (slot < topk) ? F : FS;
  const int NR = topk * F + FS;
  const int maxw = max(F, FS);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ int wcnt[kWarps];
  __shared__ int base_s;
  if (threadIdx.x == 0) base_s = 0;
  __syncthreads();
  const int64_t hrow = static_cast<int64_t>(b) * NR + static_cast<int64_t>(slot) * F;
  int32_t* out = live + (static_cast<int64_t>(b) * (topk + 1) + slot) * maxw;
  for (int g0 = 0; g0 < width / kGS; g0 += kWarps) {
    const int g = g0 + warp;
    unsigned long long m = 0ull;
    if (g < width / kGS) {
      const float v0 = load_h<HT>(h, hrow + g * kGS + lane);
      const float v1 = load_h<HT>(h, hrow + g * kGS + 32 + lane);
      m = ballot64(v0 != 0.f, v1 != 0.f);
    }
    if (lane == 0) wcnt[warp] = __popcll(m);
    __syncthreads();
    int before = base_s;
    for (int i = 0; i < warp; ++i) before += wcnt[i];
    if ((m >> lane) & 1ull) out[before + live_prefix(m, lane)] = g * kGS + lane;
    if ((m >> (lane + 32)) & 1ull) out[before + live_prefix(m, lane + 32)] = g * kGS + lane + 32;
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int i = 0; i < kWarps; ++i) t += wcnt[i];
      base_s += t;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) count[static_cast<int64_t>(b) * (topk + 1) + slot] = base_s;
}

// The staging ring per launch (measured on B200, 23 layers, z = 0.90, 192-output chunks): one
// token stages up to 1024 rows in one slot (one CTA per SM: a token's CTAs never share an
// SM); larger batches stage 256 rows in one slot (several CTAs share an SM, so a verify step
// of 3 rows runs in one wave: 24 -> 14 us a layer at B = 3, 48 -> 33 us at B = 8). Splitting the same rows into 2-8 pipelined slots measured slower at every batch
// size: the copies of a sub-batch land together, and each extra wait costs more than the
// overlap gains. HSD_DECODE_SBR / HSD_DECODE_RING force the slot rows / slot count.
inline void ring_choice(int B, int min_rb, int* sbr, int* nring) {
  static const int forced_sbr = [] { const char* e = getenv("HSD_DECODE_SBR"); return e ? atoi(e) : 0; }();
  static const int forced_ring = [] { const char* e = getenv("HSD_DECODE_RING"); return e ? atoi(e) : 0; }();
  *sbr = B == 1 ? 1024 : 256;
  *nring = 1;
  if (forced_sbr >= 64 && forced_sbr <= 1024) *sbr = forced_sbr;
  if (forced_ring >= 1 && forced_ring <= kMaxSlots) *nring = forced_ring;
  while (*sbr * *nring < min_rb || *sbr * *nring > 1024) {
    if (*sbr * *nring < min_rb) ++*nring; else --*nring;
    if (*nring > kMaxSlots) { *nring = kMaxSlots; *sbr *= 2; }
    if (*nring < 1) { *nring = 1; *sbr /= 2; }
  }
}

template <typename HT, typename ST, typename YT, int C>
int launch_decode(DecodeParams p, cudaStream_t st) {
  using Cfg = DecodeCfg<C>;
  auto kern = sparse_down_decode_kernel<HT, ST, YT, C>;
  static_assert(Cfg::MIN_RB <= Cfg::MAX_RB, "ring bounds");
  ring_choice(p.B, Cfg::MIN_RB, &p.SBR, &p.nring);
  const size_t smem = ring_offset<C>() + sizeof(uint32_t) * Cfg::NWC * p.SBR * p.nring;
  const size_t smem_max = ring_offset<C>() + sizeof(uint32_t) * Cfg::NWC * Cfg::MAX_RB;
  static int configured_device = -1;           // the attribute is set once per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem_max));
    if (e != cudaSuccess) return hsd::check_cuda(e, "hsd_sparse_down_decode: smem attribute");
    configured_device = dev;
  }
  const int nch = (p.NW + Cfg::NWC - 1) / Cfg::NWC;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nch * kCluster, p.B);
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // overlap with the previous launch
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return hsd::check_cuda(cudaLaunchKernelEx(&cfg, kern, p), "hsd_sparse_down_decode launch");
}

// Output chunk width (outputs per cluster): 256 at every batch size -- a chunk row is one
// warp's 32 words, and at D = 2688 a token is 10 full chunks and a half-width tail (88 CTAs).
// Measured per layer (B200, 23 layers, z = 0.90) against 192 (14 chunks, 24 of 32 lanes busy):
// B = 1 7.6 vs 7.7 us, B = 3 10.9 vs 14.1 us, B = 8 30.0 vs 33.0 us. HSD_DECODE_CHUNK=128 or
// 192 forces a narrower form. A token's arithmetic depends on the chunk width only (which
// words share a CTA), so with one width for all batch sizes a row of any batch (a verify row
// in particular) equals the same token decoded alone, bit for bit.
inline int chunk_choice(int) {
  static int forced = [] {
    const char* e = getenv("HSD_DECODE_CHUNK");
    return e ? atoi(e) : 0;
  }();
  if (forced == 128 || forced == 192 || forced == 256) return forced;
  return 256;
}

template <typename HT, typename ST, typename YT>
int dispatch_c(const DecodeParams& p, cudaStream_t st) {
  switch (chunk_choice(p.B)) {
    case 128: return launch_decode<HT, ST, YT, 128>(p, st);
    case 256: return launch_decode<HT, ST, YT, 256>(p, st);
  }
  return launch_decode<HT, ST, YT, 192>(p, st);
}

template <typename HT, typename ST>
int dispatch_y(int y_dtype, const DecodeParams& p, cudaStream_t st) {
  switch (y_dtype) {
    case HSD_F32: return dispatch_c<HT, ST, float>(p, st);
    case HSD_F16: return dispatch_c<HT, ST, __half>(p, st);
    case HSD_BF16: return dispatch_c<HT, ST, __nv_bfloat16>(p, st);
  }
  return hsd::set_error(HSD_ERR_DTYPE, "hsd_sparse_down_decode: y_dtype %d", y_dtype);
}

template <typename HT>
int dispatch_s(int s_dtype, int y_dtype, const DecodeParams& p, cudaStream_t st) {
  switch (s_dtype) {
    case HSD_F16: return dispatch_y<HT, __half>(y_dtype, p, st);
    case HSD_BF16: return dispatch_y<HT, __nv_bfloat16>(y_dtype, p, st);
  }
  return hsd::set_error(HSD_ERR_DTYPE, "hsd_sparse_down_decode: s_dtype %d (bf16 or f16)", s_dtype);
}

}  // namespace

namespace {

int decode_impl(const void* h, int h_dtype, const int32_t* sel, const float* gains, const uint32_t* pw,
                const void* ps, const void* pb, int s_dtype, const uint32_t* spw, const void* sps, const void* spb,
                const void* resid, void* y, int y_dtype, int B, int D, int F, int FS, int topk, int E, int loadsc,
                int all_rows, void* stream) {
  // topk == 0: the shared expert alone; FS == 0: routed experts alone (the forms the
  // expert-parallel exchange uses); the pointers of an absent part may be NULL
  if (!h || !gains || !y) return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_decode: null pointer");
  if (topk > 0 && (!sel || !pw || !ps || !pb))
    return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_decode: null routed-expert pointer");
  if (FS > 0 && (!spw || !sps || !spb))
    return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_decode: null shared-expert pointer");
  if (topk == 0) F = 64;                         // no routed columns: F is unused
  if (B < 1 || B > 65535 || D < 32 || D % 32 != 0 || F < 64 || F % 64 != 0 || FS < 0 ||
      FS % 64 != 0 || topk < 0 || (topk > 0 && E < 1) || (topk == 0 && FS == 0))
    return hsd::set_error(HSD_ERR_SHAPE,
                          "hsd_sparse_down_decode: need 1<=B<=65535, D%%32==0, F%%64==0, FS%%64==0, "
                          "topk>=0, E>=1 when topk>0, topk*F+FS>0 (got B=%d D=%d F=%d FS=%d topk=%d E=%d)",
                          B, D, F, FS, topk, E);
  const long long NR = static_cast<long long>(topk) * F + FS;
  if (NR > (1ll << 30) || static_cast<long long>(E) * F * (D / 8) > (1ll << 40))
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_sparse_down_decode: sizes too large");
  const void* ptr16[] = {h, pw, ps, pb, spw, sps, spb};
  for (const void* q : ptr16)
    if (!hsd::aligned(q, 16))
      return hsd::set_error(HSD_ERR_ALIGN, "hsd_sparse_down_decode: h and the weight pointers must be 16-byte aligned");
  DecodeParams p;
  p.h = h; p.sel = sel; p.gains = gains; p.pw = pw;
  p.ps = static_cast<const uint16_t*>(ps); p.pb = static_cast<const uint16_t*>(pb);
  p.spw = spw; p.sps = static_cast<const uint16_t*>(sps); p.spb = static_cast<const uint16_t*>(spb);
  p.resid = resid; p.y = y;
  p.B = B; p.D = D; p.F = F; p.FS = FS; p.topk = topk; p.E = E; p.loadsc = loadsc ? 1 : 0;
  p.all_rows = all_rows ? 1 : 0;
  p.NR = static_cast<int>(NR);
  p.GT = topk * (F / kGS) + FS / kGS;
  p.NW = D / 8;
  cudaStream_t st = hsd::as_stream(stream);
  switch (h_dtype) {
    case HSD_F32: return dispatch_s<float>(s_dtype, y_dtype, p, st);
    case HSD_F16: return dispatch_s<__half>(s_dtype, y_dtype, p, st);
    case HSD_BF16: return dispatch_s<__nv_bfloat16>(s_dtype, y_dtype, p, st);
  }
  return hsd::set_error(HSD_ERR_DTYPE, "hsd_sparse_down_decode: h_dtype %d", h_dtype);
}

}  // namespace

extern "C" int hsd_sparse_down_decode(const void* h, int h_dtype, const int32_t* sel,
                                      const float* gains, const uint32_t* pw, const void* ps,
                                      const void* pb, int s_dtype, const uint32_t* spw,
                                      const void* sps, const void* spb, const void* resid, void* y,
                                      int y_dtype, int B, int D, int F, int FS, int topk, int E,
                                      int loadsc, void* stream) {
  return decode_impl(h, h_dtype, sel, gains, pw, ps, pb, s_dtype, spw, sps, spb, resid, y, y_dtype, B, D, F, FS,
                     topk, E, loadsc, 0, stream);
}

extern "C" int hsd_dense_down_decode_nm(const void* h, int h_dtype, const int32_t* sel, const float* gains,
                                        const uint32_t* pw, const void* ps, const void* pb, int s_dtype,
                                        const uint32_t* spw, const void* sps, const void* spb, const void* resid,
                                        void* y, int y_dtype, int B, int D, int F, int FS, int topk, int E,
                                        void* stream) {
  return decode_impl(h, h_dtype, sel, gains, pw, ps, pb, s_dtype, spw, sps, spb, resid, y, y_dtype, B, D, F, FS,
                     topk, E, 1, 1, stream);
}

extern "C" int hsd_decode_live_rows(const void* h, int h_dtype, int32_t* live, int32_t* count, int B,
                                    int F, int FS, int topk, void* stream) {
  if (!h || !live || !count) return hsd::set_error(HSD_ERR_ARG, "hsd_decode_live_rows: null pointer");
  if (B < 1 || B > 65535 || F < 64 || F % 64 != 0 || FS < 64 || FS % 64 != 0 || topk < 1)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_decode_live_rows: bad shape");
  dim3 grid(topk + 1, B);
  cudaStream_t st = hsd::as_stream(stream);
  switch (h_dtype) {
    case HSD_F32: live_rows_kernel<float><<<grid, kLiveThreads, 0, st>>>(h, live, count, F, FS, topk); break;
    case HSD_F16: live_rows_kernel<__half><<<grid, kLiveThreads, 0, st>>>(h, live, count, F, FS, topk); break;
    case HSD_BF16:
      live_rows_kernel<__nv_bfloat16><<<grid, kLiveThreads, 0, st>>>(h, live, count, F, FS, topk);
      break;
    default: return hsd::set_error(HSD_ERR_DTYPE, "hsd_decode_live_rows: h_dtype %d", h_dtype);
  }
  return hsd::check_launch("hsd_decode_live_rows");
}
