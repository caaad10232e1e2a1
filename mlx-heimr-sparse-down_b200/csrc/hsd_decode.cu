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
//   outputs (C/2 contiguous bytes of every neuron row, one 4-byte word per lane). A
//   thread-block CLUSTER of 8 CTAs owns one (token, chunk); CTA `rank` owns groups
//   [rank*GT/8, (rank+1)*GT/8) -- at the reference shapes one routed expert or one half of
//   the shared expert (29 groups). The 8 partial outputs are summed through distributed
//   shared memory in a fixed rank order: deterministic, with no scratch memory, atomics or
//   second kernel.
//
// Per CTA: 16 group lanes (one warp each), lane L folding the CTA's groups L, L+16, L+32, ...
// in ascending order into its own 8 outputs per word, lane w of the warp owning word w of the
// chunk. A round covers 32 groups, two per warp:
//   1. the round's h values go to shared memory (16-byte cp.async pieces spread over the
//      CTA's threads) while one warp reads the groups' expert ids and gains -- one memory
//      round trip;
//   2. each warp builds its two groups' live masks (two ballots each), compacts the live rows
//      into a list (row, raw h) in shared memory, starts the cp.async copies of the first RG
//      live rows' chunks (8 lanes a row, 16 bytes a lane, four rows per instruction: the
//      memory system charges per request, not per byte), then the TMA bulk copies of the
//      live groups' scale / bias chunks on the warp's mbarrier -- one more round trip (a group
//      with more than RG live rows takes further ones: RG = 32 in the one-CTA-per-SM form used
//      at B = 1, 12 in the two-CTA-per-SM form of batches, where the group lanes' partial-chunk
//      buffer shares the staging memory);
//   3. each group's staged words and h values are read into registers, then its rows are
//      accumulated in ascending order: acc[n] += h * (8 + q_n/2), hsum += h, with
//      mixed-precision FMAs (bf16 / f16 products exact, fp32 sums); the group folds in as
//      out[n] += g * (2*s[n]*(acc[n] - 8*hsum) + b[n]*hsum) -- the reference's affine algebra
//      s * sum(h q) + b * sum(h).
// Then the 16 group lanes are reduced in shared memory in a fixed order, and each CTA pushes
// the 8 slices of its partial chunk to their owner CTAs with st.async (completing on the
// owner's mbarrier); each owner sums its slice's 8 partials in rank order.
// A token's arithmetic depends only on C: the group lanes, their fold order and both
// reduction trees are fixed, whatever the batch size, the warp count or the live counts,
// and a row dead in the token is never touched. So a row of any batch equals the same token
// decoded alone bit for bit, and the dense form (every row live) adds an exact zero where
// the sparse form skips a row: both give the same bits.
// Weights are read with an L2 evict-first policy (they are not reused by the step). The
// launch uses programmatic dependent launch: the kernel releases its dependents at once and
// waits (griddepcontrol.wait) for the previous kernel before its first read, so back-to-back
// layers overlap launch latency with the previous layer's tail. The one mbarrier wait is
// bounded (2 s of %globaltimer); running out sets HSD_ERR_TIMEOUT in the status word.
#include <cooperative_groups.h>
#include <cstdlib>

#include "hsd_common.cuh"

namespace cg = cooperative_groups;

HSD_DEFINE_STATUS(decode)

namespace {

constexpr int kCluster = 8;    // CTAs per (token, chunk)
constexpr int kGS = 64;        // quantisation group size
constexpr int kNGL = 16;       // group lanes per CTA (fixed: it sets the arithmetic)

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
};

// Shared memory of one CTA (dynamic, possibly padded by the host to limit CTAs per SM).
template <int C, int RG>
struct DecodeSmem {
  union {
    uint32_t stage[kNGL][2][RG][C / 8];         // per warp and group of a round: staged live rows
    float red[kNGL][C];                         // after the rounds: the group lanes' partial chunks
  };
  uint16_t meta[kNGL][2][2][C];                 // per warp and group of a round: scale, bias chunks
  uint32_t ch[kNGL][2][64];                     // per warp and group: h (raw bits) of the compacted live rows
  short cj[kNGL][2][64];                        //   ... and their rows
  float recv[C];                                // [rank][C/8]: the slices pushed to this CTA
  uint32_t hs[2 * kNGL][64];                    // the round's h values (raw; 64 entries of up to 4 bytes)
  int64_t grow[2 * kNGL];                       // the round's groups' first neuron rows
  int64_t gmrow[2 * kNGL];                      //   ... and scale / bias rows
  int gsrc[2 * kNGL];                           // the round's expert ids (-1 shared, -2 none)
  float ggain[2 * kNGL];                        // and gains
  unsigned long long rbar;                      // arrival of the 8 partial slices (st.async)
  unsigned long long mbar[kNGL];                // per warp: its round's scale / bias copies
};

// ---- the row arithmetic. A weight word packs the nibbles q_0..q_7 of 8 consecutive outputs
// (low nibble first). Each nibble becomes the exact value 8 + q/2 in h's precision by one shift
// and one mask-and-or -- two at a time for 16-bit h (bf16 0x4100 | q << 3, f16 0x4800 | q << 6),
// one at a time for fp32 h (0x41000000 | q << 19) -- and the row adds h * (8 + q_n/2) to acc[n]
// and h to hsum with fp32 FMAs (for 16-bit h mixed-precision ones): every product is exact and
// every sum is rounded to nearest in fp32, so acc is exactly 8x the sum of h * (1 + q/16) that
// a plain fp32 formulation would form, rounding for rounding. A group then contributes
// 2*s * (acc - 8*hsum) + b*hsum: the reference's s * sum(h q) + b * sum(h), with acc - 8*hsum
// exact (the two are within a factor 2 of each other).
template <typename HT>
struct RowMath;

template <>
struct RowMath<__nv_bfloat16> {
  // raw: the row's h as bf16 bits in the low half
  static __device__ __forceinline__ void row(float (&acc)[8], float& hsum, uint32_t raw, uint32_t w) {
    const uint32_t v0 = ((w << 3) & 0x00780078u) | 0x41004100u;   // outputs 0, 4
    const uint32_t v1 = ((w >> 1) & 0x00780078u) | 0x41004100u;   // 1, 5
    const uint32_t v2 = ((w >> 5) & 0x00780078u) | 0x41004100u;   // 2, 6
    const uint32_t v3 = ((w >> 9) & 0x00780078u) | 0x41004100u;   // 3, 7
    asm("{\n .reg .b16 a0, a1, a2, a3, a4, a5, a6, a7, hh, one;\n"
        " mov.b32 {a0, a4}, %10;\n mov.b32 {a1, a5}, %11;\n mov.b32 {a2, a6}, %12;\n mov.b32 {a3, a7}, %13;\n"
        " mov.b32 {hh, _}, %9;\n mov.b16 one, 0x3F80;\n"
        " fma.rn.f32.bf16 %0, hh, a0, %0;\n fma.rn.f32.bf16 %1, hh, a1, %1;\n"
        " fma.rn.f32.bf16 %2, hh, a2, %2;\n fma.rn.f32.bf16 %3, hh, a3, %3;\n"
        " fma.rn.f32.bf16 %4, hh, a4, %4;\n fma.rn.f32.bf16 %5, hh, a5, %5;\n"
        " fma.rn.f32.bf16 %6, hh, a6, %6;\n fma.rn.f32.bf16 %7, hh, a7, %7;\n"
        " fma.rn.f32.bf16 %8, hh, one, %8;\n}"
        : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
          "+f"(acc[7]), "+f"(hsum)
        : "r"(raw), "r"(v0), "r"(v1), "r"(v2), "r"(v3));
  }
  static __device__ __forceinline__ bool live(uint32_t raw) { return (raw & 0x7FFFu) != 0u; }
};

template <>
struct RowMath<__half> {
  static __device__ __forceinline__ void row(float (&acc)[8], float& hsum, uint32_t raw, uint32_t w) {
    const uint32_t v0 = ((w << 6) & 0x03C003C0u) | 0x48004800u;   // outputs 0, 4
    const uint32_t v1 = ((w << 2) & 0x03C003C0u) | 0x48004800u;   // 1, 5
    const uint32_t v2 = ((w >> 2) & 0x03C003C0u) | 0x48004800u;   // 2, 6
    const uint32_t v3 = ((w >> 6) & 0x03C003C0u) | 0x48004800u;   // 3, 7
    asm("{\n .reg .b16 a0, a1, a2, a3, a4, a5, a6, a7, hh, one;\n"
        " mov.b32 {a0, a4}, %10;\n mov.b32 {a1, a5}, %11;\n mov.b32 {a2, a6}, %12;\n mov.b32 {a3, a7}, %13;\n"
        " mov.b32 {hh, _}, %9;\n mov.b16 one, 0x3C00;\n"
        " fma.rn.f32.f16 %0, hh, a0, %0;\n fma.rn.f32.f16 %1, hh, a1, %1;\n"
        " fma.rn.f32.f16 %2, hh, a2, %2;\n fma.rn.f32.f16 %3, hh, a3, %3;\n"
        " fma.rn.f32.f16 %4, hh, a4, %4;\n fma.rn.f32.f16 %5, hh, a5, %5;\n"
        " fma.rn.f32.f16 %6, hh, a6, %6;\n fma.rn.f32.f16 %7, hh, a7, %7;\n"
        " fma.rn.f32.f16 %8, hh, one, %8;\n}"
        : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3]), "+f"(acc[4]), "+f"(acc[5]), "+f"(acc[6]),
          "+f"(acc[7]), "+f"(hsum)
        : "r"(raw), "r"(v0), "r"(v1), "r"(v2), "r"(v3));
  }
  static __device__ __forceinline__ bool live(uint32_t raw) { return (raw & 0x7FFFu) != 0u; }
};

template <>
struct RowMath<float> {
  template <int N>
  static __device__ __forceinline__ float q8(uint32_t w) {   // 8 + q_N / 2 as fp32
    constexpr int sh = 19 - 4 * N;
    const uint32_t m = (sh >= 0) ? (w << (sh >= 0 ? sh : 0)) : (w >> (sh < 0 ? -sh : 0));
    return __uint_as_float((m & 0x00780000u) | 0x41000000u);
  }
  static __device__ __forceinline__ void row(float (&acc)[8], float& hsum, uint32_t raw, uint32_t w) {
    const float h = __uint_as_float(raw);
    acc[0] = fmaf(h, q8<0>(w), acc[0]);
    acc[1] = fmaf(h, q8<1>(w), acc[1]);
    acc[2] = fmaf(h, q8<2>(w), acc[2]);
    acc[3] = fmaf(h, q8<3>(w), acc[3]);
    acc[4] = fmaf(h, q8<4>(w), acc[4]);
    acc[5] = fmaf(h, q8<5>(w), acc[5]);
    acc[6] = fmaf(h, q8<6>(w), acc[6]);
    acc[7] = fmaf(h, q8<7>(w), acc[7]);
    hsum += h;
  }
  static __device__ __forceinline__ bool live(uint32_t raw) { return (raw & 0x7FFFFFFFu) != 0u; }
};

// ---- memory helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t evict_normal_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}"
               ::"r"(bar), "r"(bytes) : "memory");
}
// try_wait suspends the thread until the phase completes or ~1 us passes (no hot spin).
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 1000;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// One TMA bulk copy global -> this CTA's shared memory, completing on `bar` (L2 hint).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
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
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, 1000;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait for the phase with `parity`: false after ~2 s.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > 2000000000ull) return false;
  return true;
}
// Bounded wait (cluster-scope acquire) for the phase with `parity`: false after ~2 s.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait_cluster(bar, parity))
    if (global_ns() - t0 > 2000000000ull) return false;
  return true;
}

// 16 bytes global -> this CTA's shared memory on the load/store path (cp.async, L2 hint).
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_commit_wait() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_all;" ::: "memory");
}

// Starts the copies of live-row entries [t0, t0 + RG) of a group into its stage
// ([RG][NWC] words): 8 lanes per row, 16 bytes a lane, 4 rows per warp instruction -- the memory
// system's cost is per instruction, not per byte, so a row takes a quarter of an instruction.
// Lane e holds the row offset (row * NW, in words) of list entry e in off0 and of entry 32 + e
// in off1; `rows` points at word w0 of the group's first row.
template <int RG, int NWC>
__device__ __forceinline__ void stage_rows(uint32_t stage, const uint32_t* rows, int t0, int n, int off0, int off1,
                                           int nwc, int lane, uint64_t pol) {
  const int piece = lane & 7, sub = lane >> 3;
#pragma unroll
  for (int k = 0; k < RG / 4; ++k) {
    const int e = t0 + 4 * k + sub;
    if (t0 + 4 * k < n) {                         // warp-uniform
      const int off = __shfl_sync(0xffffffffu, (t0 + 4 * k < 32) ? off0 : off1, e & 31);
      if (e < n && 4 * piece < nwc)
        cp16(stage + static_cast<uint32_t>(((4 * k + sub) * NWC + 4 * piece) * 4), rows + off + 4 * piece, pol);
    }
  }
}

// Accumulates the staged rows of entries [t0, t0 + RG), in list (ascending) order; lane e holds
// the raw h bits of entry e in hb0 and of entry 32 + e in hb1.
template <typename HT, int RG, int NWC>
__device__ __forceinline__ void consume_rows(const uint32_t* stage, int t0, int n, uint32_t hb0, uint32_t hb1,
                                             int lane, float (&acc)[8], float& hsum) {
#pragma unroll
  for (int t = 0; t < RG; ++t) {
    const int e = t0 + t;
    if (e < n) {                                  // warp-uniform
      const uint32_t hv = __shfl_sync(0xffffffffu, (t0 + t < 32) ? hb0 : hb1, e & 31);
      RowMath<HT>::row(acc, hsum, hv, stage[t * NWC + lane]);
    }
  }
}

// The same, with every entry's word and h read from shared memory first and the FMAs run back
// to back, 16 rows at a time (more registers: the one-CTA-per-SM form); chs holds the raw h of
// list entry e at e.
template <typename HT, int RG, int NWC>
__device__ __forceinline__ void consume_rows_preloaded(const uint32_t* stage, const uint32_t* chs, int t0, int n,
                                                       int lane, float (&acc)[8], float& hsum) {
  constexpr int CH = RG < 16 ? RG : 16;           // rows read into registers at a time
#pragma unroll
  for (int tb = 0; tb < RG; tb += CH) {
    if (t0 + tb >= n) break;                      // warp-uniform
    uint32_t w[CH], hv[CH];
#pragma unroll
    for (int t = 0; t < CH; ++t)
      if (tb + t < RG && t0 + tb + t < n) {       // warp-uniform; only the rows staged this round
        w[t] = stage[(tb + t) * NWC + lane];
        hv[t] = chs[t0 + tb + t];
      }
#pragma unroll
    for (int t = 0; t < CH; ++t)
      if (tb + t < RG && t0 + tb + t < n) RowMath<HT>::row(acc, hsum, hv[t], w[t]);
  }
}

template <typename HT, typename ST, typename YT, int C, int RG, int MINB>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kNGL * 32, MINB)
    sparse_down_decode_kernel(const DecodeParams p) {
  using Smem = DecodeSmem<C, RG>;
  constexpr int NWC = C / 8;                      // words of one row in a chunk
  constexpr int THREADS = kNGL * 32;
  static_assert(NWC <= 32 && NWC % 4 == 0, "a chunk row is 4..32 words, 16-byte pieces");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& S = *reinterpret_cast<Smem*>(smem_raw);
  cg::cluster_group cluster = cg::this_cluster();

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rank = static_cast<int>(cluster.block_rank());
  const int ch = blockIdx.x / kCluster;
  const int b = blockIdx.y;
  const int w0 = ch * NWC;                        // first word of this chunk
  const int nwc = min(NWC, p.NW - w0);            // words of this chunk (the tail chunk may be short)
  const bool active = lane < nwc;
  const int GF = p.F / kGS;
  const int g_lo = static_cast<int>((static_cast<long long>(rank) * p.GT) / kCluster);
  const int g_hi = static_cast<int>((static_cast<long long>(rank + 1) * p.GT) / kCluster);
  const uint32_t rbar = smem_u32(&S.rbar);
  constexpr int per = C / kCluster;               // outputs of the chunk each CTA finishes
  const uint64_t pol = evict_first_policy();
  const uint64_t hpol = evict_normal_policy();

  if (tid == 0) {
    mbar_init(rbar, 1);
    for (int w = 0; w < kNGL; ++w) mbar_init(smem_u32(&S.mbar[w]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // the 8 slices of C/8 partials that the cluster's CTAs push here complete this phase
    mbar_arrive_expect_tx(rbar, static_cast<uint32_t>(sizeof(float) * C));
  }
  __syncthreads();
  // the handshake that makes every CTA's mbarrier visible before any push (waited below)
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  // Programmatic dependent launch: let the next kernel in the stream start its launch
  // now, and wait for the previous one (which produces h / sel / gains) before reading.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  float out[8];
#pragma unroll
  for (int n = 0; n < 8; ++n) out[n] = 0.f;
  const uint32_t wbar = smem_u32(&S.mbar[warp]);
  uint32_t wphase = 0;

  const int64_t hrow = static_cast<int64_t>(b) * p.NR;
  // Round r: this warp (group lane `warp`) takes groups r0 + warp and r0 + warp + 16.
  for (int r0 = g_lo; r0 < g_hi; r0 += 2 * kNGL) {
    // ---- 1. the round's 32 groups' h values into shared memory (16-byte pieces, spread over
    //         the CTA's threads) and -- one warp for the whole CTA -- their expert ids and gains
    {
      constexpr int PIECES = 4 * static_cast<int>(sizeof(HT));   // 16-byte pieces of one group's h
      const int gi = tid / PIECES, part = tid % PIECES;
      if (gi < 2 * kNGL && r0 + gi < g_hi)
        cp16(smem_u32(&S.hs[gi][0]) + 16u * part,
             reinterpret_cast<const unsigned char*>(p.h) + (hrow + static_cast<int64_t>(r0 + gi) * kGS) * sizeof(HT) + 16 * part,
             hpol);
    }
    if (warp == 0) {
      const int g = r0 + lane;
      int src = -2;
      float gain = 0.f;
      if (g < g_hi) {
        const bool routed = g < p.topk * GF;
        const int slot = routed ? g / GF : p.topk;
        src = routed ? __ldg(p.sel + static_cast<int64_t>(b) * p.topk + slot) : -1;
        gain = __ldg(p.gains + static_cast<int64_t>(b) * (p.topk + 1) + slot);
        if (routed && (src < 0 || src >= p.E)) {
          hsd_flag_decode(HSD_ERR_INDEX);
          src = -2;
        }
      }
      S.gsrc[lane] = src;
      S.ggain[lane] = gain;
      // the group's first neuron row (in rows of its weight array) and its scale / bias row
      const int loc = (src >= 0) ? g - (g / GF) * GF : g - p.topk * GF;
      S.grow[lane] = (src >= 0) ? static_cast<int64_t>(src) * p.F + static_cast<int64_t>(loc) * kGS
                                : static_cast<int64_t>(loc) * kGS;
      S.gmrow[lane] = (src >= 0) ? static_cast<int64_t>(src) * GF + loc : loc;
    }
    cp_commit_wait();
    __syncthreads();
    // ---- 2. per group: the live mask, the compacted list of live rows (entry e: row j and its
    //         h, held by lane e % 32), the copies of the first RG live rows into the group's
    //         stage, then the scale / bias chunks -- all in flight together
    const uint32_t* rows[2];
    float gain[2];
    int n[2], off0[2], off1[2], srcs[2];
    uint32_t hv0[2], hv1[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int gi = warp + kNGL * i;              // the group's index in this round
      const int src = S.gsrc[gi];
      srcs[i] = src;
      const bool valid = src != -2;                 // (g >= g_hi is stored as -2)
      gain[i] = S.ggain[gi];
      // lane l holds entries 2l (h0) and 2l+1 (h1); even / odd live masks, bit l = entry 2l(+1)
      uint32_t h0, h1;
      if constexpr (sizeof(HT) == 4) {
        const uint2 r = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint32_t*>(&S.hs[gi][0]) + 2 * lane);
        h0 = r.x;
        h1 = r.y;
      } else {
        const uint32_t r = reinterpret_cast<const uint32_t*>(&S.hs[gi][0])[lane];
        h0 = r & 0xffffu;
        h1 = r >> 16;
      }
      const unsigned me = p.all_rows ? (valid ? 0xffffffffu : 0u) : __ballot_sync(0xffffffffu, valid && RowMath<HT>::live(h0));
      const unsigned mo = p.all_rows ? (valid ? 0xffffffffu : 0u) : __ballot_sync(0xffffffffu, valid && RowMath<HT>::live(h1));
      n[i] = __popc(me) + __popc(mo);
      rows[i] = ((src >= 0) ? p.pw : p.spw) + S.grow[gi] * p.NW + w0;   // word w0 of the group's row 0
      // compaction: row 2l+par goes to entry (live rows below it) = popc(me below l(+1)) + popc(mo below l)
      const unsigned below = (1u << lane) - 1u;     // lanes below this one
      const int eo = __popc(mo & below);
      const int ee = __popc(me & below) + eo;      // entry of row 2l
      short* cj = S.cj[warp][i];
      uint32_t* ch_ = S.ch[warp][i];
      if ((me >> lane) & 1u) {
        cj[ee] = static_cast<short>(2 * lane);
        ch_[ee] = h0;
      }
      if ((mo >> lane) & 1u) {
        const int e1 = ee + static_cast<int>((me >> lane) & 1u);          // entry of row 2l+1
        cj[e1] = static_cast<short>(2 * lane + 1);
        ch_[e1] = h1;
      }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      off0[i] = (lane < n[i]) ? S.cj[warp][i][lane] * p.NW : 0;
      off1[i] = (lane + 32 < n[i]) ? S.cj[warp][i][lane + 32] * p.NW : 0;
      hv0[i] = (lane < n[i]) ? S.ch[warp][i][lane] : 0u;
      hv1[i] = (lane + 32 < n[i]) ? S.ch[warp][i][lane + 32] : 0u;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i)
      stage_rows<RG, NWC>(smem_u32(&S.stage[warp][i][0][0]), rows[i], 0, n[i], off0[i], off1[i], nwc, lane, pol);
    // the live groups' scale and bias chunks: TMA bulk copies (nwc*16 bytes each) into the
    // warp's area, completing on the warp's mbarrier, beside the load/store path the rows use
    const uint32_t mbytes = static_cast<uint32_t>(nwc) * 16;
    const bool ml0 = p.loadsc && n[0] != 0, ml1 = p.loadsc && n[1] != 0;
    const uint32_t wbytes = ((ml0 ? 1u : 0u) + (ml1 ? 1u : 0u)) * 2 * mbytes;
    if (wbytes != 0 && lane < 4) {
      const int i = lane >> 1, sb = lane & 1;
      if (lane == 0) mbar_arrive_expect_tx(wbar, wbytes);
      __syncwarp(0xfu);
      if (i == 0 ? ml0 : ml1) {
        const int src = i == 0 ? srcs[0] : srcs[1];
        const int64_t mrow = S.gmrow[warp + kNGL * i];
        const uint16_t* base = (src >= 0) ? (sb ? p.pb : p.ps) : (sb ? p.spb : p.sps);
        bulk_g2s(&S.meta[warp][i][sb][0], base + mrow * p.D + static_cast<int64_t>(w0) * 8, mbytes, wbar, pol);
      }
    }
    cp_commit_wait();
    __syncwarp();
    bool meta_in = wbytes == 0;                  // warp-uniform
    // ---- 3. accumulate and fold, the lane's groups in ascending order
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      if (n[i] == 0) continue;                    // warp-uniform
      float acc[8], hsum = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = 0.f;
      if constexpr (MINB == 1)
        consume_rows_preloaded<HT, RG, NWC>(&S.stage[warp][i][0][0], &S.ch[warp][i][0], 0, n[i], lane, acc, hsum);
      else
        consume_rows<HT, RG, NWC>(&S.stage[warp][i][0][0], 0, n[i], hv0[i], hv1[i], lane, acc, hsum);
      for (int t0 = RG; t0 < n[i]; t0 += RG) {     // groups with more than RG live rows
        __syncwarp();
        stage_rows<RG, NWC>(smem_u32(&S.stage[warp][i][0][0]), rows[i], t0, n[i], off0[i], off1[i], nwc, lane, pol);
        cp_commit_wait();
        __syncwarp();
        if constexpr (MINB == 1)
          consume_rows_preloaded<HT, RG, NWC>(&S.stage[warp][i][0][0], &S.ch[warp][i][0], t0, n[i], lane, acc, hsum);
        else
          consume_rows<HT, RG, NWC>(&S.stage[warp][i][0][0], t0, n[i], hv0[i], hv1[i], lane, acc, hsum);
      }
      if (!meta_in) {                            // the chunks are needed from the first fold on
        if (!mbar_wait_bounded(wbar, wphase)) {
          if (lane == 0) hsd_flag_decode(HSD_ERR_TIMEOUT);
          mbar_wait_bounded(wbar, wphase);       // once more for the copies still in flight
        }
        wphase ^= 1u;
        meta_in = true;
      }
      const float h8 = 8.f * hsum;               // exact
      if (active) {
        if (p.loadsc) {
          const uint4 s4 = *reinterpret_cast<const uint4*>(&S.meta[warp][i][0][lane * 8]);
          const uint4 b4 = *reinterpret_cast<const uint4*>(&S.meta[warp][i][1][lane * 8]);
          const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
          const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float sc = hsd::bits16_to_f32<ST>(static_cast<uint16_t>(sw[k >> 1] >> (16 * (k & 1))));
            const float bi = hsd::bits16_to_f32<ST>(static_cast<uint16_t>(bw[k >> 1] >> (16 * (k & 1))));
            out[k] = fmaf(gain[i], fmaf(2.f * sc, acc[k] - h8, bi * hsum), out[k]);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 8; ++k) out[k] = fmaf(gain[i], fmaf(2.f, acc[k] - h8, hsum), out[k]);
        }
      }
    }
    __syncthreads();                             // the round's shared tables are rewritten next
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // before the next round's bulk copies
  }

  // ---- 4. the 16 group lanes' partial chunks into shared memory
  if (lane < NWC) {
    *reinterpret_cast<float4*>(&S.red[warp][lane * 8]) = make_float4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<float4*>(&S.red[warp][lane * 8 + 4]) = make_float4(out[4], out[5], out[6], out[7]);
  }
  __syncthreads();
  // ---- 5. the cluster's 8 partials: slice r of every CTA's chunk goes to CTA r (st.async,
  //         completing on CTA r's rbar), which sums the 8 slices in rank order; each output's
  //         partial is pushed by the thread that sums its 16 group lanes
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");   // every rbar is initialised
  for (int o = tid; o < C; o += THREADS) {       // 4 partial sums of 4 lanes, then their sum
    float q4[4];
#pragma unroll
    for (int qd = 0; qd < 4; ++qd) {
      float a = 0.f;
#pragma unroll
      for (int L = 4 * qd; L < 4 * qd + 4; ++L) a += S.red[L][o];
      q4[qd] = a;
    }
    const float part = (q4[0] + q4[1]) + (q4[2] + q4[3]);
    const int dst = o / per;
    st_async_f32(mapa_u32(smem_u32(&S.recv[rank * per + (o - dst * per)]), dst), part, mapa_u32(rbar, dst));
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

// ---- active-index sets (hsd/decode.py:86-101): per (token, slot) the ascending nonzero
//      indices, by warp ballots and prefix popcounts

// Live mask of 64 h values (entry j read by lane j % 32) with two ballots.
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

template <typename HT>
__device__ __forceinline__ float load_h(const void* h, int64_t idx) {
  return hsd::to_f32<HT>(reinterpret_cast<const HT*>(h)[idx]);
}

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

// Launch shape. Chunks of C = 256 outputs (a chunk row is one warp's 32 words; at D = 2688
// a token is 10 full chunks and a half-width tail, 88 CTAs per token) and 16 warps per CTA.
// One token loads up to 32 live rows of a group per round trip (128 registers, one CTA per
// SM); a batch up to 12 (64 registers: two CTAs per SM, so a 3-row verify step runs in one
// wave). HSD_DECODE_RG (16: the one-token form, 8: the batch form) and HSD_DECODE_SMEM
// (dynamic shared memory in bytes, to limit the CTAs per SM) override the choice;
// HSD_DECODE_CHUNK (128, 160, 192, 256) the chunk width.
// None of them changes a token's arithmetic.
int env_int(const char* name) {
  const char* e = getenv(name);
  return e ? atoi(e) : 0;
}

template <typename HT, typename ST, typename YT, int C, int RG, int MINB>
int launch_decode(const DecodeParams& p, cudaStream_t st) {
  auto kern = sparse_down_decode_kernel<HT, ST, YT, C, RG, MINB>;
  static const int forced_smem = env_int("HSD_DECODE_SMEM");
  size_t smem = sizeof(DecodeSmem<C, RG>);
  if (forced_smem > 0 && static_cast<size_t>(forced_smem) > smem) smem = static_cast<size_t>(forced_smem);
  if (smem > 227 * 1024) smem = 227 * 1024;
  static int configured_device = -1;           // the attribute is set once per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return hsd::check_cuda(e, "hsd_sparse_down_decode: smem attribute");
    configured_device = dev;
  }
  const int nch = (p.NW + C / 8 - 1) / (C / 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nch * kCluster, p.B);
  cfg.blockDim = dim3(kNGL * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // overlap with the previous launch
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return hsd::check_cuda(cudaLaunchKernelEx(&cfg, kern, p), "hsd_sparse_down_decode launch");
}

template <typename HT, typename ST, typename YT, int C>
int dispatch_rg(const DecodeParams& p, cudaStream_t st) {
  static const int forced = env_int("HSD_DECODE_RG");
  const int rg = (forced == 8 || forced == 16) ? forced : (p.B == 1 ? 16 : 8);
  if (rg == 16) return launch_decode<HT, ST, YT, C, 32, 1>(p, st);
  return launch_decode<HT, ST, YT, C, 12, 2>(p, st);
}

template <typename HT, typename ST, typename YT>
int dispatch_c(const DecodeParams& p, cudaStream_t st) {
  static const int forced = env_int("HSD_DECODE_CHUNK");
  switch (forced) {
    case 128: return dispatch_rg<HT, ST, YT, 128>(p, st);
    case 160: return dispatch_rg<HT, ST, YT, 160>(p, st);
    case 192: return dispatch_rg<HT, ST, YT, 192>(p, st);
  }
  return dispatch_rg<HT, ST, YT, 256>(p, st);
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
