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
  qmma_kernel<MODE, ST><<<grid, kThreads, smem, st>>>(p);
  return hsd::check_launch(who);
}

}  // namespace

namespace hsd {

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
  return s_dtype == HSD_BF16 ? launch_qmma<kQLinear, __nv_bfloat16>(p, p.shared_tiles, st, "hsd_qlinear_decode")
                             : launch_qmma<kQLinear, __half>(p, p.shared_tiles, st, "hsd_qlinear_decode");
}

}  // namespace hsd
