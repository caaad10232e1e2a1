// 4-bit g64 matrix-vector products of decode rows on the tensor cores (warp-level
// mma.m16n8k16, fp16 operands, fp32 accumulation): the up projections of the MoE front end
// (hsd/model.py:110-121) and the model's plain 4-bit linears, for up to 8 token rows at once.
//
// A warp computes 16 weight rows (the MMA's M) against up to 8 token rows (its N) over a
// slice of the reduction axis; the 8 warps of a block take the 64-groups g = warp, warp+8, ..
// and their partial outputs are summed in warp order through shared memory (deterministic).
//
//   A fragment (weights): the checkpoint layout packs 8 consecutive columns per word, low
//     nibble first. The MMA's k slots are permuted inside every 8 columns so that slot pair
//     (2c, 2c+1) holds columns (c, c+4): one mask-and-or of the word shifted by 4c gives the
//     fp16 pair (1024 + q_c, 1024 + q_{c+4}) exactly, minus 1024 gives the integers q.
//   B fragment (tokens): the token rows in fp16, stored in shared memory already in the
//     permuted order, two 32-bit pairs per (token, 16 columns, c).
//   Per 64-group the four MMAs give sum q x over the group (exact fp16 products, fp32
//     accumulation in the tensor core); the group adds s * that + b * sum x.
//
// The token values are rounded to fp16 (bf16 inputs are exact in fp16 inside its range).
// An output element depends only on its weight row and its token row, so a token's result
// does not depend on the other tokens of the launch.
#include <algorithm>
#include <cstdlib>

#include "hsd_common.cuh"

HSD_DEFINE_STATUS(qmma)

#ifndef HSD_QMMA_GB
#define HSD_QMMA_GB 4        // 64-groups a warp has in flight at once
#endif

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 16;          // weight rows per block (the MMA's M)
constexpr int kCols = 8;           // token rows per MMA (the MMA's N)

enum QMode { kQUp = 0, kQLinear = 1 };

struct QParams {
  const void* x;        // [B, red] token rows (bf16 / f16 / f32), row stride x_stride
  int64_t x_stride;
  int x_dtype;
  const int32_t* sel;   // up form: [B, topk]
  const uint32_t* uw;   // up form routed: [E, F, red/8]
  const uint16_t* us;
  const uint16_t* ub;
  const uint32_t* w;    // shared expert (up form) or the linear's weights: [rows, red/8]
  const uint16_t* s;
  const uint16_t* b;
  const void* resid;    // linear form: [B, rows] (y dtype) or null
  void* y;
  int y_dtype;
  int B, red, F, FS, topk, E;
  int routed_tiles;     // up form: B * topk * ceil(F / 16)
  int shared_tiles;     // ceil(rows_shared / 16)
  int col_groups;       // ceil(B / 8) for the multi-token tiles
};

__device__ __forceinline__ float load_f(const void* x, int dtype, int64_t i) {
  switch (dtype) {
    case HSD_F32: return reinterpret_cast<const float*>(x)[i];
    case HSD_F16: return __half2float(reinterpret_cast<const __half*>(x)[i]);
    default: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
  }
}

__device__ __forceinline__ void store_f(void* y, int dtype, int64_t i, float v) {
  switch (dtype) {
    case HSD_F32: reinterpret_cast<float*>(y)[i] = v; break;
    case HSD_F16: reinterpret_cast<__half*>(y)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<__nv_bfloat16*>(y)[i] = __float2bfloat16_rn(v); break;
  }
}

// fp16 pair (q_c, q_{c+4}) of word w, shift = 4c: exact small integers
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int shift) {
  const uint32_t h = ((w >> shift) & 0x000F000Fu) | 0x64006400u;       // (1024 + q_c, 1024 + q_{c+4})
  uint32_t r;
  asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64006400u));
  return r;
}

__device__ __forceinline__ void mma16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Shared memory: xh [kc cols][red/16 chunks][4 c] of uint2 (b0, b1) with a 32-byte skew per
// column, xsum [kc cols][red/64] fp32 group sums, part [8 warps][16 rows][8 cols] fp32;
// kc = min(B, 8) columns are staged.
__host__ __device__ constexpr int xh_col_stride_u2(int red) { return (red / 16) * 4 + 4; }

template <int MODE, typename ST>
__global__ void __launch_bounds__(kThreads) qmma_kernel(const QParams p) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int red = p.red, NG = red / 64, WR = red / 8, GR = red / 64;
  const int cs = xh_col_stride_u2(red);
  const int kc = min(p.B, kCols);                   // token columns staged (shared-memory layout)
  uint2* xh = reinterpret_cast<uint2*>(smem);
  float* xsum = reinterpret_cast<float*>(smem + static_cast<size_t>(kc) * cs * sizeof(uint2));
  float* part = xsum + kc * NG;

  // ---- which 16 weight rows, which token rows (columns)
  const uint32_t* W;
  const uint16_t* S;
  const uint16_t* Bz;
  int rows, r0, col0, ncols;
  int64_t y_base, y_col_stride;       // y index = y_base + col * y_col_stride + row
  int t = blockIdx.x;
  bool bad = false;
  if (MODE == kQUp && t < p.routed_tiles) {
    const int tiles_f = (p.F + kTile - 1) / kTile;
    const int bk = t / tiles_f;                       // (token, slot) = (bk / topk, bk % topk)
    const int bi = bk / p.topk, k = bk % p.topk;
    r0 = (t % tiles_f) * kTile;
    rows = p.F;
    const int e = p.sel[bi * p.topk + k];
    bad = e < 0 || e >= p.E;
    const int ee = bad ? 0 : e;
    W = p.uw + static_cast<int64_t>(ee) * p.F * WR;
    S = p.us + static_cast<int64_t>(ee) * p.F * GR;
    Bz = p.ub + static_cast<int64_t>(ee) * p.F * GR;
    col0 = bi;
    ncols = 1;
    y_base = static_cast<int64_t>(bi) * (p.topk * p.F + p.FS) + static_cast<int64_t>(k) * p.F;
    y_col_stride = 0;
  } else {
    if (MODE == kQUp) t -= p.routed_tiles;
    const int tile = t / p.col_groups, cg = t % p.col_groups;
    r0 = tile * kTile;
    rows = p.FS;                                      // the shared expert's / the linear's rows
    W = p.w;
    S = p.s;
    Bz = p.b;
    col0 = cg * kCols;
    ncols = min(kCols, p.B - col0);
    if (MODE == kQUp) {
      y_base = static_cast<int64_t>(p.topk) * p.F;
      y_col_stride = static_cast<int64_t>(p.topk) * p.F + p.FS;
    } else {
      y_base = 0;
      y_col_stride = p.FS;
    }
  }
  if (bad) {                                           // an expert id outside [0, E): zeros
    if (tid == 0) hsd_flag_qmma(HSD_ERR_INDEX);
    for (int i = tid; i < kTile; i += kThreads)
      if (r0 + i < rows) store_f(p.y, p.y_dtype, y_base + static_cast<int64_t>(col0) * y_col_stride + r0 + i, 0.f);
    return;
  }

  // ---- this warp's rows r0 + g and r0 + g + 8; its first group's words and scales are
  // requested before the token is staged, so the two latencies overlap
  const int ra = min(r0 + g, rows - 1), rb = min(r0 + g + 8, rows - 1);
  const uint32_t* wa = W + static_cast<int64_t>(ra) * WR;
  const uint32_t* wb = W + static_cast<int64_t>(rb) * WR;
  // the warp's groups in batches of kGB, every load of a batch in flight at once
  constexpr int kGB = HSD_QMMA_GB;
  uint4 bw[kGB][4];
  uint16_t bq[kGB][4];
  auto fetch = [&](int gr, uint4* wv, uint16_t* qv) {
    wv[0] = hsd::ldg_nc_v4(wa + gr * 8);
    wv[1] = hsd::ldg_nc_v4(wa + gr * 8 + 4);
    wv[2] = hsd::ldg_nc_v4(wb + gr * 8);
    wv[3] = hsd::ldg_nc_v4(wb + gr * 8 + 4);
    qv[0] = __ldg(S + static_cast<int64_t>(ra) * GR + gr);
    qv[1] = __ldg(S + static_cast<int64_t>(rb) * GR + gr);
    qv[2] = __ldg(Bz + static_cast<int64_t>(ra) * GR + gr);
    qv[3] = __ldg(Bz + static_cast<int64_t>(rb) * GR + gr);
  };
  auto fetch_batch = [&](int base) {
#pragma unroll
    for (int i = 0; i < kGB; ++i) {
      const int gr = base + i * kWarps;
      if (gr < NG) fetch(gr, bw[i], bq[i]);
    }
  };
  fetch_batch(warp);

  // ---- the token rows in fp16, permuted for the B fragment, and their fp32 group sums: one
  // thread per (column, 16 values), a 16-value sum per thread, a group sum over 4 lanes
  const int nch = red / 16;
  for (int t0 = 0; t0 < ncols * nch; t0 += kThreads) {
    const int t = t0 + tid;
    float csum = 0.f;
    if (t < ncols * nch) {
      const int col = t / nch, ch = t % nch;
      const int64_t xb = static_cast<int64_t>(col0 + col) * p.x_stride + ch * 16;
      __half hv[16];
      if (p.x_dtype == HSD_BF16 && (reinterpret_cast<uintptr_t>(static_cast<const uint16_t*>(p.x) + xb) & 15) == 0) {
        const uint4 r0v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + xb));
        const uint4 r1v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + xb) + 1);
        const uint32_t wd[8] = {r0v.x, r0v.y, r0v.z, r0v.w, r1v.x, r1v.y, r1v.z, r1v.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          hv[2 * i] = __float2half_rn(__uint_as_float(wd[i] << 16));
          hv[2 * i + 1] = __float2half_rn(__uint_as_float(wd[i] & 0xffff0000u));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) hv[i] = __float2half_rn(load_f(p.x, p.x_dtype, xb + i));
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint2 v;
        v.x = static_cast<uint32_t>(__half_as_ushort(hv[cc])) | (static_cast<uint32_t>(__half_as_ushort(hv[cc + 4])) << 16);
        v.y = static_cast<uint32_t>(__half_as_ushort(hv[cc + 8])) | (static_cast<uint32_t>(__half_as_ushort(hv[cc + 12])) << 16);
        xh[col * cs + ch * 4 + cc] = v;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) csum += __half2float(hv[i]);
    }
    // the 4 chunks of a group are 4 adjacent threads (nch is a multiple of 4)
    csum += __shfl_xor_sync(0xffffffffu, csum, 1);
    csum += __shfl_xor_sync(0xffffffffu, csum, 2);
    if (t < ncols * nch && (t & 3) == 0) xsum[(t / nch) * NG + (t % nch) / 4] = csum;
  }
  __syncthreads();

  // token columns past ncols read column ncols-1 (their outputs are never stored)
  const int gq = min(g, ncols - 1);
  float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;      // (ra, col 2c), (ra, 2c+1), (rb, 2c), (rb, 2c+1)
  const int sh = 4 * c;
  for (int base = warp; base < NG; base += kGB * kWarps) {
    if (base != warp) fetch_batch(base);
#pragma unroll
    for (int i = 0; i < kGB; ++i) {
      const int gr = base + i * kWarps;
      if (gr >= NG) break;
      const uint4* cw = bw[i];
      const uint16_t* cq = bq[i];
      const uint32_t wa_[8] = {cw[0].x, cw[0].y, cw[0].z, cw[0].w, cw[1].x, cw[1].y, cw[1].z, cw[1].w};
      const uint32_t wb_[8] = {cw[2].x, cw[2].y, cw[2].z, cw[2].w, cw[3].x, cw[3].y, cw[3].z, cw[3].w};
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 4; ++j) {                  // 16 columns: words 2j (k 0-7) and 2j+1 (k 8-15)
        const uint32_t a[4] = {nib_pair(wa_[2 * j], sh), nib_pair(wb_[2 * j], sh), nib_pair(wa_[2 * j + 1], sh),
                               nib_pair(wb_[2 * j + 1], sh)};
        const uint2 bx = xh[gq * cs + (gr * 4 + j) * 4 + c];
        mma16816(d, a, bx.x, bx.y);
      }
      const float sa = hsd::bits16_to_f32<ST>(cq[0]), sb = hsd::bits16_to_f32<ST>(cq[1]);
      const float ba = hsd::bits16_to_f32<ST>(cq[2]), bb = hsd::bits16_to_f32<ST>(cq[3]);
      const float xs0 = xsum[min(2 * c, ncols - 1) * NG + gr], xs1 = xsum[min(2 * c + 1, ncols - 1) * NG + gr];
      y0 = fmaf(sa, d[0], fmaf(ba, xs0, y0));
      y1 = fmaf(sa, d[1], fmaf(ba, xs1, y1));
      y2 = fmaf(sb, d[2], fmaf(bb, xs0, y2));
      y3 = fmaf(sb, d[3], fmaf(bb, xs1, y3));
    }
  }

  // ---- the 8 warps' partials, summed in warp order
  float* pw = part + warp * (kTile * kCols);
  pw[g * kCols + 2 * c] = y0;
  pw[g * kCols + 2 * c + 1] = y1;
  pw[(g + 8) * kCols + 2 * c] = y2;
  pw[(g + 8) * kCols + 2 * c + 1] = y3;
  __syncthreads();
  for (int i = tid; i < kTile * kCols; i += kThreads) {
    const int row = i / kCols, col = i % kCols;
    if (col >= ncols || r0 + row >= rows) continue;
    float acc = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < kWarps; ++w8) acc += part[w8 * (kTile * kCols) + i];
    const int64_t yi = y_base + static_cast<int64_t>(col0 + col) * y_col_stride + r0 + row;
    if (MODE == kQUp) {
      const float v = fmaxf(acc, 0.f);
      store_f(p.y, p.y_dtype, yi, v * v);
    } else {
      const float rv = p.resid ? load_f(p.resid, p.y_dtype, yi) : 0.f;
      store_f(p.y, p.y_dtype, yi, rv + acc);
    }
  }
}

// ---- the streaming form (B <= 8, every row count a multiple of 16): one persistent block
// per SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...; a tile's 16 weight rows and
// their scales / biases arrive by TMA bulk copies into a ring of `nst` shared-memory stages
// (one mbarrier each), so the weights stream while earlier tiles compute, and the token rows
// are staged once per block. 16 warps split a tile's 64-groups (g = warp, warp+16, ..., two
// at a time for independent MMA chains) and their partials are summed in warp order.
// Measured on B200 (CUDA-graph replay, weights rotated through HBM): the 131072 x 2688 lm_head
// at one row 79 us (2.5 TB/s) against 128 us for the one-tile-per-block form; per tile, one
// bulk copy of the 16 contiguous rows beat 16 copies of padded rows (TMA time per copy), and
// 16 warps with two groups in flight beat 8 warps with one.
constexpr int kStMax = 8;
constexpr int kSWarps = 16;
constexpr int kSThreads = kSWarps * 32;

__device__ __forceinline__ uint32_t q_smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool q_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait (~2 s of %globaltimer); false when it ran out.
__device__ __forceinline__ bool q_wait_bounded(uint32_t bar, uint32_t parity) {
  if (q_try_wait(bar, parity)) return true;
  uint64_t t0, t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (!q_try_wait(bar, parity)) {
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > 2000000000ull) return false;
  }
  return true;
}
__device__ __forceinline__ void q_bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                           uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}

struct QTile {
  const uint32_t* W;   // the tile's first weight row
  const uint16_t* S;   // its scale rows ([16][red/64])
  const uint16_t* Bz;  // its bias rows
  int col0, ncols;
  int64_t y_base, y_col_stride;
  bool bad;
};

// Tile t of the launch (the same tiles as qmma_kernel with one column group, B <= 8).
template <int MODE>
__device__ __forceinline__ QTile q_tile(const QParams& p, int t, const int* sel_s) {
  QTile q;
  const int WR = p.red / 8, GR = p.red / 64;
  if (MODE == kQUp && t < p.routed_tiles) {
    const int tiles_f = p.F / kTile;
    const int bk = t / tiles_f;
    const int bi = bk / p.topk, k = bk % p.topk;
    const int r0 = (t % tiles_f) * kTile;
    const int e = sel_s[bi * p.topk + k];
    q.bad = e < 0 || e >= p.E;
    const int64_t row = static_cast<int64_t>(q.bad ? 0 : e) * p.F + r0;
    q.W = p.uw + row * WR;
    q.S = p.us + row * GR;
    q.Bz = p.ub + row * GR;
    q.col0 = bi;
    q.ncols = 1;
    q.y_base = static_cast<int64_t>(bi) * (p.topk * p.F + p.FS) + static_cast<int64_t>(k) * p.F + r0;
    q.y_col_stride = 0;
  } else {
    if (MODE == kQUp) t -= p.routed_tiles;
    const int r0 = t * kTile;
    q.bad = false;
    q.W = p.w + static_cast<int64_t>(r0) * WR;
    q.S = p.s + static_cast<int64_t>(r0) * GR;
    q.Bz = p.b + static_cast<int64_t>(r0) * GR;
    q.col0 = 0;
    q.ncols = p.B;
    if (MODE == kQUp) {
      q.y_base = static_cast<int64_t>(p.topk) * p.F + r0;
      q.y_col_stride = static_cast<int64_t>(p.topk) * p.F + p.FS;
    } else {
      q.y_base = r0;
      q.y_col_stride = p.FS;
    }
  }
  return q;
}

struct QStreamCfg {
  int ntiles, nst;
  uint32_t stage_bytes;  // one stage: 16 weight rows of red/8 words, then scales, biases
  uint32_t off_stages;   // byte offsets in dynamic shared memory
  uint32_t off_bars, off_sel, off_part;
};

template <int MODE, typename ST>
__global__ void __launch_bounds__(kSThreads, 1) qstream_kernel(const QParams p, const QStreamCfg sc) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int red = p.red, NG = red / 64, WR = red / 8, GR = red / 64;
  const int cs = xh_col_stride_u2(red);
  const int kc = p.B;                                 // every token column is staged (B <= 8)
  uint2* xh = reinterpret_cast<uint2*>(smem);
  float* xsum = reinterpret_cast<float*>(smem + static_cast<size_t>(kc) * cs * sizeof(uint2));
  float* part = reinterpret_cast<float*>(smem + sc.off_part);    // [2][8 warps][16][8]
  int* sel_s = reinterpret_cast<int*>(smem + sc.off_sel);
  unsigned char* stages = smem + sc.off_stages;
  const uint32_t bar0 = q_smem_u32(smem + sc.off_bars);
  const uint32_t tile_bytes = 16u * static_cast<uint32_t>(WR) * 4u + 2u * 16u * static_cast<uint32_t>(GR) * 2u;
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));

  // programmatic dependent launch: a linear's first weight tiles are requested before the
  // wait for the previous kernel (weights are never written by the step); the up form's
  // tiles depend on the routing, so it waits first
  hsd::pdl_launch_dependents();
  if (MODE == kQUp) {
    hsd::pdl_wait();
    for (int i = tid; i < p.B * p.topk; i += kSThreads) sel_s[i] = p.sel[i];
  }
  if (tid == 0)
    for (int s = 0; s < sc.nst; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar0 + 8u * s) : "memory");
  __syncthreads();

  // the producer: tile t into stage s (its 16 weight rows, scale rows and bias rows: 3 copies)
  auto issue = [&](int t, int s) {
    const QTile q = q_tile<MODE>(p, t, sel_s);
    const uint32_t st = q_smem_u32(stages + static_cast<size_t>(s) * sc.stage_bytes);
    const uint32_t bar = bar0 + 8u * s;
    asm volatile("{\n .reg .b64 x;\n mbarrier.arrive.expect_tx.shared::cta.b64 x, [%0], %1;\n}"
                 ::"r"(bar), "r"(tile_bytes) : "memory");
    q_bulk_g2s(st, q.W, static_cast<uint32_t>(kTile * WR) * 4u, bar, pol);   // 16 contiguous rows
    const uint32_t sb = st + static_cast<uint32_t>(kTile * WR) * 4u;
    q_bulk_g2s(sb, q.S, 16u * GR * 2u, bar, pol);
    q_bulk_g2s(sb + 16u * GR * 2u, q.Bz, 16u * GR * 2u, bar, pol);
  };
  if (tid == 0)
    for (int i = 0; i < sc.nst; ++i) {
      const int t = blockIdx.x + i * gridDim.x;
      if (t < sc.ntiles) issue(t, i);
    }
  if (MODE != kQUp) hsd::pdl_wait();               // x and y from here on

  // ---- the token rows in fp16, permuted for the B fragment, and their fp32 group sums
  const int nch = red / 16;
  for (int t0 = 0; t0 < kc * nch; t0 += kSThreads) {
    const int t = t0 + tid;
    float csum = 0.f;
    if (t < kc * nch) {
      const int col = t / nch, ch = t % nch;
      const int64_t xb = static_cast<int64_t>(col) * p.x_stride + ch * 16;
      __half hv[16];
      if (p.x_dtype == HSD_BF16 && (reinterpret_cast<uintptr_t>(static_cast<const uint16_t*>(p.x) + xb) & 15) == 0) {
        const uint4 r0v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + xb));
        const uint4 r1v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + xb) + 1);
        const uint32_t wd[8] = {r0v.x, r0v.y, r0v.z, r0v.w, r1v.x, r1v.y, r1v.z, r1v.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          hv[2 * i] = __float2half_rn(__uint_as_float(wd[i] << 16));
          hv[2 * i + 1] = __float2half_rn(__uint_as_float(wd[i] & 0xffff0000u));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) hv[i] = __float2half_rn(load_f(p.x, p.x_dtype, xb + i));
      }
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint2 v;
        v.x = static_cast<uint32_t>(__half_as_ushort(hv[cc])) | (static_cast<uint32_t>(__half_as_ushort(hv[cc + 4])) << 16);
        v.y = static_cast<uint32_t>(__half_as_ushort(hv[cc + 8])) | (static_cast<uint32_t>(__half_as_ushort(hv[cc + 12])) << 16);
        xh[col * cs + ch * 4 + cc] = v;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) csum += __half2float(hv[i]);
    }
    csum += __shfl_xor_sync(0xffffffffu, csum, 1);
    csum += __shfl_xor_sync(0xffffffffu, csum, 2);
    if (t < kc * nch && (t & 3) == 0) xsum[(t / nch) * NG + (t % nch) / 4] = csum;
  }
  __syncthreads();

  const int sh = 4 * c;
  for (int i = 0;; ++i) {
    const int t = blockIdx.x + i * gridDim.x;
    if (t >= sc.ntiles) break;
    const int s = i % sc.nst;
    const QTile q = q_tile<MODE>(p, t, sel_s);
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(stages + static_cast<size_t>(s) * sc.stage_bytes);
    const uint16_t* sS = reinterpret_cast<const uint16_t*>(sw + kTile * WR);
    const uint16_t* sB = sS + 16 * GR;
    if (!q_wait_bounded(bar0 + 8u * s, static_cast<uint32_t>(i / sc.nst) & 1u)) {
      if (tid == 0) hsd_flag_qmma(HSD_ERR_TIMEOUT);
      q_wait_bounded(bar0 + 8u * s, static_cast<uint32_t>(i / sc.nst) & 1u);   // copies in flight
    }
    const int gq = q.col0 + min(g, q.ncols - 1);
    const int xc0 = q.col0 + min(2 * c, q.ncols - 1), xc1 = q.col0 + min(2 * c + 1, q.ncols - 1);
    float y0 = 0.f, y1 = 0.f, y2 = 0.f, y3 = 0.f;
#pragma unroll 2
    for (int gr = warp; gr < NG; gr += kSWarps) {
      const uint4 a0 = *reinterpret_cast<const uint4*>(sw + g * WR + gr * 8);
      const uint4 a1 = *reinterpret_cast<const uint4*>(sw + g * WR + gr * 8 + 4);
      const uint4 b0 = *reinterpret_cast<const uint4*>(sw + (g + 8) * WR + gr * 8);
      const uint4 b1 = *reinterpret_cast<const uint4*>(sw + (g + 8) * WR + gr * 8 + 4);
      const uint32_t wa_[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const uint32_t wb_[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t a[4] = {nib_pair(wa_[2 * j], sh), nib_pair(wb_[2 * j], sh), nib_pair(wa_[2 * j + 1], sh),
                               nib_pair(wb_[2 * j + 1], sh)};
        const uint2 bx = xh[gq * cs + (gr * 4 + j) * 4 + c];
        mma16816(d, a, bx.x, bx.y);
      }
      const float sa = hsd::bits16_to_f32<ST>(sS[g * GR + gr]), sb = hsd::bits16_to_f32<ST>(sS[(g + 8) * GR + gr]);
      const float ba = hsd::bits16_to_f32<ST>(sB[g * GR + gr]), bb = hsd::bits16_to_f32<ST>(sB[(g + 8) * GR + gr]);
      const float xs0 = xsum[xc0 * NG + gr], xs1 = xsum[xc1 * NG + gr];
      y0 = fmaf(sa, d[0], fmaf(ba, xs0, y0));
      y1 = fmaf(sa, d[1], fmaf(ba, xs1, y1));
      y2 = fmaf(sb, d[2], fmaf(bb, xs0, y2));
      y3 = fmaf(sb, d[3], fmaf(bb, xs1, y3));
    }
    float* pw = part + ((i & 1) * kSWarps + warp) * (kTile * kCols);
    pw[g * kCols + 2 * c] = y0;
    pw[g * kCols + 2 * c + 1] = y1;
    pw[(g + 8) * kCols + 2 * c] = y2;
    pw[(g + 8) * kCols + 2 * c + 1] = y3;
    __syncthreads();                                  // stage s read by every warp; partials written
    if (tid == 0 && t + sc.nst * static_cast<int>(gridDim.x) < sc.ntiles) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(t + sc.nst * gridDim.x, s);
    }
    const float* pt = part + (i & 1) * kSWarps * (kTile * kCols);
    if (q.bad && tid == 0) hsd_flag_qmma(HSD_ERR_INDEX);
    for (int e = tid; e < kTile * kCols; e += kSThreads) {
      const int row = e / kCols, col = e % kCols;
      if (col >= q.ncols) continue;
      float acc = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < kSWarps; ++w8) acc += pt[w8 * (kTile * kCols) + e];
      const int64_t yi = q.y_base + static_cast<int64_t>(q.col0 + col) * q.y_col_stride + row;
      if (MODE == kQUp) {
        const float v = q.bad ? 0.f : fmaxf(acc, 0.f);
        store_f(p.y, p.y_dtype, yi, v * v);
      } else {
        const float rv = p.resid ? load_f(p.resid, p.y_dtype, yi) : 0.f;
        store_f(p.y, p.y_dtype, yi, rv + acc);
      }
    }
  }
}

// The streaming form's shared-memory plan: false when it does not apply (B > 8, a row count
// that is not a multiple of 16, or fewer than two stages fit), or when HSD_QMMA_STREAM=0.
bool qstream_plan(const QParams& p, int ntiles, QStreamCfg* sc, size_t* smem) {
  static const bool disabled = [] { const char* e = getenv("HSD_QMMA_STREAM"); return e && atoi(e) == 0; }();
  if (disabled || p.B < 1 || p.B > kCols || p.red % 64 != 0 || ntiles < 1) return false;
  if ((p.routed_tiles > 0 && p.F % kTile != 0) || p.FS % kTile != 0) return false;
  const size_t WR = p.red / 8, GR = p.red / 64;
  size_t off = static_cast<size_t>(p.B) * xh_col_stride_u2(p.red) * sizeof(uint2) + p.B * GR * sizeof(float);
  off = (off + 15) / 16 * 16;
  sc->off_part = static_cast<uint32_t>(off);
  off += 2 * kSWarps * kTile * kCols * sizeof(float);
  sc->off_sel = static_cast<uint32_t>(off);
  off += 64 * sizeof(int);
  sc->off_bars = static_cast<uint32_t>(off);
  off += kStMax * 8;
  off = (off + 127) / 128 * 128;
  sc->off_stages = static_cast<uint32_t>(off);
  const size_t stage = ((kTile * WR * 4 + 2 * kTile * GR * 2) + 127) / 128 * 128;
  constexpr size_t kBudget = 200 * 1024;
  if (off + 2 * stage > kBudget || p.B * p.topk > 64) return false;
  const int nst = static_cast<int>(std::min<size_t>(kStMax, (kBudget - off) / stage));
  sc->ntiles = ntiles;
  sc->nst = nst;
  sc->stage_bytes = static_cast<uint32_t>(stage);
  *smem = off + nst * stage;
  return true;
}

template <int MODE, typename ST>
int launch_qstream(const QParams& p, const QStreamCfg& sc, size_t smem, cudaStream_t st, const char* who) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms < 1) sms = 1;
  }
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(qstream_kernel<MODE, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024);
    if (e != cudaSuccess) return hsd::check_cuda(e, who);
    configured = true;
  }
  const int grid = std::min(sc.ntiles, sms);
  hsd::launch_pdl(qstream_kernel<MODE, ST>, dim3(grid), dim3(kSThreads), smem, st, p, sc);
  return hsd::check_launch(who);
}

// shared memory for `cols` token columns (min(B, 8))
size_t qmma_smem(int red, int cols) {
  return static_cast<size_t>(cols) * xh_col_stride_u2(red) * sizeof(uint2) + cols * (red / 64) * sizeof(float) +
         kWarps * kTile * kCols * sizeof(float);
}

template <int MODE, typename ST>
int launch_qmma(const QParams& p, int grid, cudaStream_t st, const char* who) {
  const size_t smem = qmma_smem(p.red, min(p.B, kCols));
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(qmma_kernel<MODE, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return hsd::check_cuda(e, who);
  }
  hsd::launch_pdl(qmma_kernel<MODE, ST>, dim3(grid), dim3(kThreads), smem, st, p);
  return hsd::check_launch(who);
}

}  // namespace

namespace hsd {

inline bool aligned16(const void* q) { return q == nullptr || (reinterpret_cast<uintptr_t>(q) & 15) == 0; }

// The MoE up projections with relu2 on the tensor cores (hsd_moe_up_decode's arguments).
int qmma_moe_up(const void* x, int x_dtype, int64_t x_stride, const int32_t* sel, const uint32_t* uw,
                const void* us, const void* ub, int s_dtype, const uint32_t* suw, const void* sus, const void* sub,
                void* h, int h_dtype, int B, int D, int F, int FS, int topk, int E, cudaStream_t st) {
  QParams p;
  p.x = x; p.x_stride = x_stride; p.x_dtype = x_dtype; p.sel = sel;
  p.uw = uw; p.us = static_cast<const uint16_t*>(us); p.ub = static_cast<const uint16_t*>(ub);
  p.w = suw; p.s = static_cast<const uint16_t*>(sus); p.b = static_cast<const uint16_t*>(sub);
  p.resid = nullptr; p.y = h; p.y_dtype = h_dtype;
  p.B = B; p.red = D; p.F = F; p.FS = FS; p.topk = topk; p.E = E;
  p.routed_tiles = topk > 0 ? B * topk * ((F + kTile - 1) / kTile) : 0;
  p.col_groups = (B + kCols - 1) / kCols;
  p.shared_tiles = FS > 0 ? ((FS + kTile - 1) / kTile) * p.col_groups : 0;
  const int64_t grid = static_cast<int64_t>(p.routed_tiles) + p.shared_tiles;
  if (grid > 0x7fffffff) return set_error(HSD_ERR_SHAPE, "hsd_moe_up_decode: grid too large");
  QStreamCfg sc;
  size_t smem = 0;
  const bool al = aligned16(uw) && aligned16(us) && aligned16(ub) && aligned16(suw) && aligned16(sus) &&
                  aligned16(sub);
  if (al && qstream_plan(p, static_cast<int>(grid), &sc, &smem))
    return s_dtype == HSD_BF16 ? launch_qstream<kQUp, __nv_bfloat16>(p, sc, smem, st, "hsd_moe_up_decode")
                               : launch_qstream<kQUp, __half>(p, sc, smem, st, "hsd_moe_up_decode");
  return s_dtype == HSD_BF16 ? launch_qmma<kQUp, __nv_bfloat16>(p, static_cast<int>(grid), st, "hsd_moe_up_decode")
                             : launch_qmma<kQUp, __half>(p, static_cast<int>(grid), st, "hsd_moe_up_decode");
}

// A plain 4-bit linear on the tensor cores (hsd_qlinear_decode's arguments).
int qmma_linear(const void* x, int x_dtype, int64_t x_stride, const uint32_t* w, const void* s, const void* b,
                int s_dtype, const void* resid, void* y, int y_dtype, int B, int in_f, int out_f, cudaStream_t st) {
  QParams p;
  p.x = x; p.x_stride = x_stride; p.x_dtype = x_dtype; p.sel = nullptr;
  p.uw = nullptr; p.us = nullptr; p.ub = nullptr;
  p.w = w; p.s = static_cast<const uint16_t*>(s); p.b = static_cast<const uint16_t*>(b);
  p.resid = resid; p.y = y; p.y_dtype = y_dtype;
  p.B = B; p.red = in_f; p.F = 0; p.FS = out_f; p.topk = 0; p.E = 0;
  p.routed_tiles = 0;
  p.col_groups = (B + kCols - 1) / kCols;
  p.shared_tiles = ((out_f + kTile - 1) / kTile) * p.col_groups;
  if (static_cast<int64_t>(p.shared_tiles) > 0x7fffffff) return set_error(HSD_ERR_SHAPE, "hsd_qlinear_decode: grid too large");
  QStreamCfg sc;
  size_t smem = 0;
  if (aligned16(w) && aligned16(s) && aligned16(b) && qstream_plan(p, p.shared_tiles, &sc, &smem))
    return s_dtype == HSD_BF16 ? launch_qstream<kQLinear, __nv_bfloat16>(p, sc, smem, st, "hsd_qlinear_decode")
                               : launch_qstream<kQLinear, __half>(p, sc, smem, st, "hsd_qlinear_decode");
  return s_dtype == HSD_BF16 ? launch_qmma<kQLinear, __nv_bfloat16>(p, p.shared_tiles, st, "hsd_qlinear_decode")
                             : launch_qmma<kQLinear, __half>(p, p.shared_tiles, st, "hsd_qlinear_decode");
}

}  // namespace hsd
