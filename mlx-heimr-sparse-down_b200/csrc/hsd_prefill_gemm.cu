// Grouped-by-expert prefill GEMM on the neuron-major layout with 5th-generation tensor
// cores (tcgen05 / TMEM), sm_100a (hsd/prefill.py:119-222 is the reference's Metal version).
//
// One work item = (tile of 128 slots of one expert, block of 192 output columns). For the
// item's expert, over K-tiles of 64 neurons (exactly one quantisation group each):
//   A [128 slots x 64] fp16   the gathered h rows (hc), TMA 2D load, 128-byte swizzle (K-major)
//   W [64 neurons x 24 words] the packed 4-bit rows of the block, TMA 2D load (no swizzle)
//   s, b [192]                the group's scales / biases of the block, two bulk copies
//   B [64 x 192] fp16         dequantised in shared memory by 12 warps, s*q + b with one
//                             fp16 rounding (half2 FMA), written MN-major with the 128-byte
//                             swizzle the tensor core reads
//   D [128 x 192] fp32 += A . B, tcgen05.mma.cta_group::1.kind::f16 issued by one thread,
//                             accumulated in TMEM (two 256-column buffers: the epilogue of one
//                             item overlaps the MMAs of the next)
// Epilogue (4 warps, one TMEM lane quadrant each): tcgen05.ld 32 columns at a time, times the
// slot's routing gain, stored to part[token*(topk+1) + k, :] (fp32), or -- expert parallelism --
// to the slot's row of its home GPU's partial buffer through a per-slot pointer table (plain
// stores over NVLink). A separate fixed-order reduce sums the topk+1 partial rows of each token.
//
// Warp roles (31 warps): 0 TMA producer, 1 MMA issuer (and TMEM owner), 2-5 epilogue, 6 scale
// converter (bf16 -> fp16 pairs), 7-30 dequantisation. A / packed-W stages ring through 5
// buffers, dequantised B through 3, each with full / empty mbarriers (measured: 5 / 3 / 24
// dequant warps 2 % faster than 7 / 2 / 12 at 2048-token chunks, the same bits). Every mbarrier
// wait is bounded (2 s of %globaltimer); running out sets HSD_ERR_TIMEOUT in the status word
// and the role stops; TMEM is freed after a bounded wait for the epilogue. No multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "hsd_common.cuh"
#include "hsd_prefill.cuh"

HSD_DEFINE_STATUS(gemm)

namespace {

#ifndef HSD_GEMM_BN
#define HSD_GEMM_BN 192
#endif
constexpr int BM = 128, BN = HSD_GEMM_BN, BK = 64;
#ifndef HSD_GEMM_STAGES
#define HSD_GEMM_STAGES 5
#endif
#ifndef HSD_GEMM_BSTAGES
#define HSD_GEMM_BSTAGES 3
#endif
constexpr int STAGES = HSD_GEMM_STAGES;                       // A / packed-W / scale stages in flight
constexpr int BSTAGES = HSD_GEMM_BSTAGES;                     // dequantised B buffers
#ifndef HSD_GEMM_DQ_WARPS
#define HSD_GEMM_DQ_WARPS 24
#endif
constexpr int DQ_WARPS = HSD_GEMM_DQ_WARPS;
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_EPI0 = 2, WARP_CONV = 6, WARP_DQ0 = 7;
constexpr int NWARPS = WARP_DQ0 + DQ_WARPS, THREADS = NWARPS * 32;
constexpr int DQ_THREADS = DQ_WARPS * 32;
constexpr int WPB = BN / 8;                                   // packed words per row of a block (24)
constexpr uint32_t A_BYTES = BM * BK * 2;                     // 16 KB
constexpr uint32_t B_BYTES = BK * BN * 2;                     // 24 KB
constexpr uint32_t W_BYTES = BK * WPB * 4;                    // 6 KB
constexpr uint32_t SB_BYTES = 2 * BN * 2;                     // 768 B (scales then biases)
constexpr uint32_t TX_BYTES = A_BYTES + W_BYTES + SB_BYTES;
constexpr uint32_t OFF_A = 0;
constexpr uint32_t OFF_B = OFF_A + STAGES * A_BYTES;
constexpr uint32_t OFF_W = OFF_B + BSTAGES * B_BYTES;
constexpr uint32_t OFF_SB = OFF_W + STAGES * W_BYTES;
constexpr uint32_t OFF_SBH = OFF_SB + STAGES * SB_BYTES;      // fp16 scale / bias pairs per stage
constexpr uint32_t OFF_BAR = OFF_SBH + STAGES * SB_BYTES;     // 8-byte barriers
// full_tma[STAGES], empty[STAGES], bfull[BSTAGES], bempty[BSTAGES], acc_full[2], acc_empty[2], done,
// conv[STAGES]
constexpr int NBARS = 2 * STAGES + 2 * BSTAGES + 2 + 2 + 1 + STAGES;
constexpr uint32_t OFF_TMEM = OFF_BAR + NBARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_TMEM + 16 + 1024;         // + slack for 1024-byte alignment
constexpr uint32_t TMEM_COLS = 512, ACC_COLS = 256;
constexpr uint32_t B_LBO = (BK / 8) * 1024;                   // B: bytes between 64-column atoms
static_assert(B_BYTES == (BN / 64) * B_LBO, "B tile = N atoms x K groups");
static_assert(BN % 64 == 0 && BN <= 256 && BN % 16 == 0, "UMMA N");
static_assert(OFF_B % 1024 == 0 && A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "swizzled tiles 1024-aligned");
static_assert((BK * WPB) % DQ_THREADS == 0 && DQ_THREADS % WPB == 0,
              "dequant: a whole number of units per thread, one fixed word per thread");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");

// instruction descriptor: D f32, A f16 (K-major), B f16 (MN-major), N = 192, M = 128
constexpr uint32_t IDESC = (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) |
                           (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);

struct GemmParams {
  const int32_t* tile_e;
  const int32_t* tile_slot;
  const float* gains;
  const uint16_t* ps;
  const uint16_t* pb;
  const uint16_t* sps;
  const uint16_t* spb;
  float* part;
  float* const* row_dst;   // optional: routed slot s's output row is row_dst[s] (another GPU's memory allowed)
  float* shared_out;       // optional: the shared expert's row of token t is shared_out + t * D
  const uint8_t* kmask;    // [NT][KG] live-K-tile bytes from the gather (KG: kmax / 64 rounded up to 8)
  int NT, T, D, F, FS, topk, E, nnt, KG;
};

// Whether a role processes K-tile kt of a tile: when the tile has a nonzero A value in it, or
// when it is the tile's last K-tile and none was processed before (an all-zero tile still
// writes its accumulator: zeros). `done` counts the K-tiles processed so far; `word` caches
// the 8 mask bytes of kt's 8-aligned block (rows of KG bytes, KG a multiple of 8). Every role
// applies the same rule to the same bytes, so all roles walk the same K-tiles.
__device__ __forceinline__ bool kt_run(const GemmParams& p, int tile, int kt, int KT, int done, uint64_t& word) {
  if ((kt & 7) == 0)
    word = __ldg(reinterpret_cast<const unsigned long long*>(p.kmask + static_cast<int64_t>(tile) * p.KG + kt));
  return ((word >> (8 * (kt & 7))) & 0xFFu) != 0 || (kt == KT - 1 && done == 0);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(bar) : "memory");
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
// Bounded wait for the phase with `parity`; false (and HSD_ERR_TIMEOUT recorded) after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > 2000000000ull) {
      hsd_flag_gemm(HSD_ERR_TIMEOUT);
      return false;
    }
  return true;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
// shared-memory matrix descriptor, 128-byte swizzle, Blackwell version bits
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accum) {
  asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
               ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accum) : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16-bit scale / bias bits -> fp16 bits (exact for bf16 values in fp16's normal range)
template <typename ST> __device__ __forceinline__ uint32_t pair_to_h2(uint32_t two);
template <> __device__ __forceinline__ uint32_t pair_to_h2<__half>(uint32_t two) { return two; }
template <> __device__ __forceinline__ uint32_t pair_to_h2<__nv_bfloat16>(uint32_t two) {
  const float lo = __uint_as_float(two << 16), hi = __uint_as_float(two & 0xFFFF0000u);
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace

namespace {

__device__ __forceinline__ __half2 u32_as_h2(uint32_t x) { return *reinterpret_cast<const __half2*>(&x); }
__device__ __forceinline__ uint32_t h2_as_u32(__half2 x) { return *reinterpret_cast<const uint32_t*>(&x); }

template <typename ST>
__global__ void __launch_bounds__(THREADS, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w,
                        const __grid_constant__ CUtensorMap map_ws, const GemmParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;            // swizzled tiles need 1024-byte alignment
  unsigned char* gbase = smem_raw + (base - raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bars = base + OFF_BAR;
  auto bar_full_tma = [&](int s) { return bars + 8u * s; };
  auto bar_empty = [&](int s) { return bars + 8u * (STAGES + s); };
  auto bar_bfull = [&](int j) { return bars + 8u * (2 * STAGES + j); };
  auto bar_bempty = [&](int j) { return bars + 8u * (2 * STAGES + BSTAGES + j); };
  auto bar_acc_full = [&](int a) { return bars + 8u * (2 * STAGES + 2 * BSTAGES + a); };
  auto bar_acc_empty = [&](int a) { return bars + 8u * (2 * STAGES + 2 * BSTAGES + 2 + a); };
  const uint32_t bar_done = bars + 8u * (2 * STAGES + 2 * BSTAGES + 4);
  auto bar_conv = [&](int s) { return bars + 8u * (2 * STAGES + 2 * BSTAGES + 5 + s); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_TMEM);

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full_tma(s), 1);
      mbar_init(bar_empty(s), 1);
      mbar_init(bar_conv(s), 1);
    }
    for (int j = 0; j < BSTAGES; ++j) {
      mbar_init(bar_bfull(j), DQ_WARPS);
      mbar_init(bar_bempty(j), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(bar_acc_full(a), 1);
      mbar_init(bar_acc_empty(a), 4);
    }
    mbar_init(bar_done, 4);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_ws)) : "memory");
  }
  if (warp == WARP_MMA) {                                  // the whole warp allocates TMEM
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int nitems = p.NT * p.nnt;
  const int GF = p.F / BK, GFS = p.FS / BK;

  if (warp == WARP_TMA) {
    // ---- producer: A tile, packed W rows, the group's scale / bias slices
    if (lane == 0) {
      int stage = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
        const int tile = it / p.nnt, nt = it - tile * p.nnt;
        const int e = p.tile_e[tile];
        if (e < 0) continue;
        const bool shared = e >= p.E;
        const int KT = shared ? GFS : GF;              // 0 for shared tiles when FS == 0: skipped
        int done = 0;
        uint64_t mword = 0;
        for (int kt = 0; kt < KT; ++kt) {
          if (!kt_run(p, tile, kt, KT, done, mword)) continue;   // only zeros to multiply
          ++done;
          if (!mbar_wait(bar_empty(stage), ph ^ 1u)) {
            ok = false;
            break;
          }
          const uint32_t fb = bar_full_tma(stage);
          mbar_arrive_expect_tx(fb, TX_BYTES);
          tma_load_2d(base + OFF_A + stage * A_BYTES, &map_a, fb, kt * BK, tile * BM);
          if (shared) tma_load_2d(base + OFF_W + stage * W_BYTES, &map_ws, fb, nt * WPB, kt * BK);
          else tma_load_2d(base + OFF_W + stage * W_BYTES, &map_w, fb, nt * WPB, e * p.F + kt * BK);
          const int64_t grow = shared ? kt : static_cast<int64_t>(e) * GF + kt;
          const int64_t mo = grow * p.D + static_cast<int64_t>(nt) * BN;
          bulk_load(base + OFF_SB + stage * SB_BYTES, (shared ? p.sps : p.ps) + mo, BN * 2, fb);
          bulk_load(base + OFF_SB + stage * SB_BYTES + BN * 2, (shared ? p.spb : p.pb) + mo, BN * 2, fb);
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == WARP_MMA) {
    // ---- MMA issuer: one thread, accumulators in TMEM (two buffers)
    if (lane == 0) {
      int stage = 0, acc = 0, bj = 0;
      uint32_t ph = 0, aph = 0, bph = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
        const int tile = it / p.nnt;
        const int e = p.tile_e[tile];
        if (e < 0) continue;
        const int KT = (e >= p.E) ? GFS : GF;
        if (KT == 0) continue;
        if (!mbar_wait(bar_acc_empty(acc), aph ^ 1u)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc) * ACC_COLS;
        uint32_t accum = 0;                                // the item's first MMA overwrites
        int done = 0;
        uint64_t mword = 0;
        for (int kt = 0; kt < KT; ++kt) {
          if (!kt_run(p, tile, kt, KT, done, mword)) continue;
          ++done;
          if (!mbar_wait(bar_full_tma(stage), ph) || !mbar_wait(bar_bfull(bj), bph)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = base + OFF_A + stage * A_BYTES, b0 = base + OFF_B + bj * B_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            umma_f16(d, sw128_desc(a0 + kk * 32, 16, 1024), sw128_desc(b0 + kk * 2048, B_LBO, 1024), accum);
            accum = 1u;
          }
          umma_commit(bar_empty(stage));                   // frees the A / W stage when these MMAs finish
          umma_commit(bar_bempty(bj));                     // and the B buffer
          if (++stage == STAGES) {
            stage = 0;
            ph ^= 1u;
          }
          if (++bj == BSTAGES) {
            bj = 0;
            bph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(bar_acc_full(acc));                    // the item's accumulator is complete
        if (++acc == 2) {
          acc = 0;
          aph ^= 1u;
        }
      }
    }
    __syncwarp();
    mbar_wait(bar_done, 0);                                // the epilogue is done with TMEM
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
  } else if (warp < WARP_EPI0 + 4) {
    // ---- epilogue: TMEM lane quadrant (warp % 4), gain, fp32 partial rows
    const int q = warp & 3;
    const int m = 32 * q + lane;
    int acc = 0;
    uint32_t aph = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
      const int tile = it / p.nnt, nt = it - tile * p.nnt;
      const int e = p.tile_e[tile];
      if (e < 0 || ((e >= p.E) ? GFS : GF) == 0) continue;
      if (!mbar_wait(bar_acc_full(acc), aph)) break;
      tc_fence_after();
      const int s = p.tile_slot[static_cast<int64_t>(tile) * BM + m];
      int64_t row = -1;
      float g = 0.f;
      float* out_row = nullptr;
      if (s >= 0) {
        row = (e >= p.E) ? static_cast<int64_t>(s) * (p.topk + 1) + p.topk
                         : static_cast<int64_t>(s / p.topk) * (p.topk + 1) + (s % p.topk);
        g = __ldg(p.gains + row);
        out_row = (e >= p.E) ? (p.shared_out ? p.shared_out + static_cast<int64_t>(s) * p.D : p.part + row * p.D)
                             : (p.row_dst ? p.row_dst[s] : p.part + row * p.D);
      }
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(acc) * ACC_COLS;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(taddr + c0, v);
        if (out_row) {
          float* dst = out_row + static_cast<int64_t>(nt) * BN + c0;
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) = make_float4(v[i] * g, v[i + 1] * g, v[i + 2] * g, v[i + 3] * g);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_acc_empty(acc));
      if (++acc == 2) {
        acc = 0;
        aph ^= 1u;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_done);
  } else if (warp == WARP_CONV) {
    // ---- scales / biases of each stage -> fp16 pairs (n, n+4) in the dequant's order
    int stage = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
      const int tile = it / p.nnt;
      const int e = p.tile_e[tile];
      if (e < 0) continue;
      const int KT = (e >= p.E) ? GFS : GF;
      int done = 0;
      uint64_t mword = 0;
      for (int kt = 0; kt < KT; ++kt) {
        if (!kt_run(p, tile, kt, KT, done, mword)) continue;
        ++done;
        // (the stage's previous fp16 pairs were read before its previous MMAs, which came
        // before the producer refilled it: the full barrier alone orders the overwrite)
        if (!mbar_wait(bar_full_tma(stage), ph)) {
          ok = false;
          break;
        }
        const uint32_t* sb = reinterpret_cast<const uint32_t*>(gbase + OFF_SB + stage * SB_BYTES);
        uint32_t* sbh = reinterpret_cast<uint32_t*>(gbase + OFF_SBH + stage * SB_BYTES);
        for (int t = lane; t < 2 * WPB; t += 32) {          // t < 24: scales of word t, else biases
          const int wd = t % WPB, which = t / WPB;
          // 8 values of word wd: (0,1)(2,3)(4,5)(6,7) -> pairs (0,4)(1,5)(2,6)(3,7), one 16-byte
          // load and store per lane (consecutive lanes, consecutive 16-byte chunks)
          const uint4 v = *reinterpret_cast<const uint4*>(sb + which * (BN / 2) + wd * 4);
          *reinterpret_cast<uint4*>(sbh + which * (BN / 2) + wd * 4) =
              make_uint4(pair_to_h2<ST>(__byte_perm(v.x, v.z, 0x5410)), pair_to_h2<ST>(__byte_perm(v.x, v.z, 0x7632)),
                         pair_to_h2<ST>(__byte_perm(v.y, v.w, 0x5410)), pair_to_h2<ST>(__byte_perm(v.y, v.w, 0x7632)));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_conv(stage));
        if (++stage == STAGES) {
          stage = 0;
          ph ^= 1u;
        }
      }
    }
  } else {
    // ---- dequantisation: packed rows -> fp16 B tile, MN-major, 128-byte swizzle.
    // Thread d owns word w = d % 24 of every row it touches (rows k0, k0+16, k0+32, k0+48,
    // k0 = d / 24), so its 8 scales and 8 biases are read once per K-tile. A word's nibbles
    // become fp16 pairs (n, n+4) with one mask-and-or each (1024 + q, exact), minus 1024,
    // times the pair's scales plus biases (one fp16 rounding), then byte permutes restore
    // output order.
    const int d = tid - WARP_DQ0 * 32;                      // 0 .. DQ_THREADS-1
    const int w = d % WPB, k0 = d / WPB;
    int stage = 0, bj = 0;
    uint32_t ph = 0, bph = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
      const int tile = it / p.nnt;
      const int e = p.tile_e[tile];
      if (e < 0) continue;
      const int KT = (e >= p.E) ? GFS : GF;
      int done = 0;
      uint64_t mword = 0;
      for (int kt = 0; kt < KT; ++kt) {
        if (!kt_run(p, tile, kt, KT, done, mword)) continue;
        ++done;
        if (!mbar_wait(bar_full_tma(stage), ph) || !mbar_wait(bar_conv(stage), ph) ||
            !mbar_wait(bar_bempty(bj), bph ^ 1u)) {
          ok = false;
          break;
        }
        const uint32_t* wr = reinterpret_cast<const uint32_t*>(gbase + OFF_W + stage * W_BYTES);
        const uint32_t* sbh = reinterpret_cast<const uint32_t*>(gbase + OFF_SBH + stage * SB_BYTES);
        unsigned char* bt = gbase + OFF_B + bj * B_BYTES;
        const uint4 s4 = *reinterpret_cast<const uint4*>(sbh + w * 4);
        const uint4 b4 = *reinterpret_cast<const uint4*>(sbh + BN / 2 + w * 4);
#pragma unroll
        for (int i = 0; i < BK / (DQ_THREADS / WPB); ++i) {
          const int k = k0 + (DQ_THREADS / WPB) * i;       // neuron row of the K-tile
          const uint32_t qw = wr[k * WPB + w];
          const __half2 m1024 = u32_as_h2(0x64006400u);
          const __half2 v0 = __hfma2(__hsub2(u32_as_h2((qw & 0x000F000Fu) | 0x64006400u), m1024), u32_as_h2(s4.x), u32_as_h2(b4.x));
          const __half2 v1 = __hfma2(__hsub2(u32_as_h2(((qw >> 4) & 0x000F000Fu) | 0x64006400u), m1024), u32_as_h2(s4.y), u32_as_h2(b4.y));
          const __half2 v2 = __hfma2(__hsub2(u32_as_h2(((qw >> 8) & 0x000F000Fu) | 0x64006400u), m1024), u32_as_h2(s4.z), u32_as_h2(b4.z));
          const __half2 v3 = __hfma2(__hsub2(u32_as_h2(((qw >> 12) & 0x000F000Fu) | 0x64006400u), m1024), u32_as_h2(s4.w), u32_as_h2(b4.w));
          // v_j = outputs (j, j+4): outputs (0,1), (2,3), (4,5), (6,7)
          const uint32_t o0 = __byte_perm(h2_as_u32(v0), h2_as_u32(v1), 0x5410);
          const uint32_t o1 = __byte_perm(h2_as_u32(v2), h2_as_u32(v3), 0x5410);
          const uint32_t o2 = __byte_perm(h2_as_u32(v0), h2_as_u32(v1), 0x7632);
          const uint32_t o3 = __byte_perm(h2_as_u32(v2), h2_as_u32(v3), 0x7632);
          const uint32_t off = static_cast<uint32_t>(w >> 3) * B_LBO + static_cast<uint32_t>(k >> 3) * 1024u +
                               static_cast<uint32_t>(k & 7) * 128u +
                               (static_cast<uint32_t>((w & 7) ^ (k & 7)) << 4);
          *reinterpret_cast<uint4*>(bt + off) = make_uint4(o0, o1, o2, o3);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> tensor core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_bfull(bj));
        if (++stage == STAGES) {
          stage = 0;
          ph ^= 1u;
        }
        if (++bj == BSTAGES) {
          bj = 0;
          bph ^= 1u;
        }
      }
    }
  }
}

}  // namespace

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
              uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle sw, const char* what) {
  auto enc = tensor_map_encoder();
  if (!enc) return hsd::set_error(HSD_ERR_CUDA, "prefill gemm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return hsd::set_error(HSD_ERR_CUDA, "prefill gemm: tensor map (%s) error %d", what, (int)r);
  return HSD_OK;
}

template <typename ST>
int launch_typed(const CUtensorMap& ma, const CUtensorMap& mw, const CUtensorMap& mws, const GemmParams& p,
                 cudaStream_t st) {
  static int configured_device = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(prefill_gemm_kernel<ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(SMEM_BYTES));
    if (e != cudaSuccess) return hsd::check_cuda(e, "prefill gemm: smem attribute");
    configured_device = dev;
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int nitems = p.NT * p.nnt;
  const int grid = nitems < sms ? nitems : sms;
  if (grid < 1) return HSD_OK;
  prefill_gemm_kernel<ST><<<grid, THREADS, SMEM_BYTES, st>>>(ma, mw, mws, p);
  return hsd::check_launch("prefill gemm");
}

}  // namespace

namespace hsd {

int launch_prefill_gemm(const __half* hc, int kmax, const int32_t* tile_e, const int32_t* tile_slot, int NT,
                        const uint8_t* kmask, const float* gains, const uint32_t* pw, const void* ps, const void* pb, int s_dtype,
                        const uint32_t* spw, const void* sps, const void* spb, float* part, int T, int D,
                        int F, int FS, int topk, int E, cudaStream_t st, float* const* row_dst,
                        float* shared_out) {
  if (D % BN != 0 || F % BK != 0 || FS < 0 || FS % BK != 0 || kmax % BK != 0)
    return set_error(HSD_ERR_SHAPE, "prefill gemm: need D %% %d == 0, F and FS %% 64 == 0 (D=%d F=%d FS=%d)", BN,
                     D, F, FS);
  CUtensorMap ma, mw, mws;
  int rc = encode_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hc, static_cast<uint64_t>(kmax),
                     static_cast<uint64_t>(NT) * BM, static_cast<uint64_t>(kmax) * 2, BK, BM,
                     CU_TENSOR_MAP_SWIZZLE_128B, "A");
  if (rc) return rc;
  rc = encode_2d(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, pw, static_cast<uint64_t>(D / 8),
                 static_cast<uint64_t>(E) * F, static_cast<uint64_t>(D / 8) * 4, WPB, BK, CU_TENSOR_MAP_SWIZZLE_NONE,
                 "W");
  if (rc) return rc;
  // (with FS == 0 there are no shared tiles to load: the routed map stands in, unused)
  rc = FS > 0 ? encode_2d(&mws, CU_TENSOR_MAP_DATA_TYPE_UINT32, spw, static_cast<uint64_t>(D / 8),
                          static_cast<uint64_t>(FS), static_cast<uint64_t>(D / 8) * 4, WPB, BK,
                          CU_TENSOR_MAP_SWIZZLE_NONE, "Ws")
              : (mws = mw, HSD_OK);
  if (rc) return rc;
  GemmParams p;
  p.tile_e = tile_e;
  p.tile_slot = tile_slot;
  p.gains = gains;
  p.ps = static_cast<const uint16_t*>(ps);
  p.pb = static_cast<const uint16_t*>(pb);
  p.sps = static_cast<const uint16_t*>(sps);
  p.spb = static_cast<const uint16_t*>(spb);
  p.part = part;
  p.row_dst = row_dst;
  p.shared_out = shared_out;
  p.kmask = kmask;
  p.KG = (kmax / BK + 7) / 8 * 8;
  p.NT = NT;
  p.T = T;
  p.D = D;
  p.F = F;
  p.FS = FS;
  p.topk = topk;
  p.E = E;
  p.nnt = D / BN;
  switch (s_dtype) {
    case HSD_BF16: return launch_typed<__nv_bfloat16>(ma, mw, mws, p, st);
    case HSD_F16: return launch_typed<__half>(ma, mw, mws, p, st);
  }
  return set_error(HSD_ERR_DTYPE, "prefill gemm: s_dtype %d (bf16 or f16)", s_dtype);
}

}  // namespace hsd
