// 4-bit g64 matrix-vector products over the selected experts of decode rows, on the
// checkpoint layout (rows = outputs, 4-bit groups of 64 along the reduction axis). The C-ABI
// entry points of this file:
//
//   hsd_moe_up_decode   the MoE front end's up projections with ReLU^2 (the reference's
//                       hsd/model.py:110-121), and
//   hsd_qlinear_decode  the model's plain 4-bit linears -- both computed on the tensor
//                       cores by csrc/hsd_qmma.cu;
//   hsd_dense_down_decode  the stock (dense) MoE down projection the sparse kernel is
//          compared with (hsd/model.py:132-133 decode_dense, mlx gather_qmm of fc2 and the
//          shared down_proj), by the fp32 CUDA-core kernel below: part k reads its own slice
//          h[b, k*F ..], every weight of the selected experts is read, the part's gain is
//          applied and the fp32 partial rows [B, topk+1, D] are summed in slot order (+ resid)
//          by the prefill path's reduce kernel, so the dense output is deterministic.
//
// The CUDA-core kernel: one block per (token b, part, tile of 16 output rows), part k < topk
// the routed expert sel[b, k] and part topk the shared expert (1176 blocks for one token of
// the reference shapes). Each warp owns one row (16 warps a block, so many warps are in
// flight per SM to hide the memory latency). Lane l reads the 16-byte pieces l, l+32, l+64,
// .. of a row (a piece = 32 consecutive columns = half a 64-group), so every row is read by
// one coalesced sweep and each weight byte once; all of the row's pieces, scales and biases
// are loaded before any arithmetic.
//
// Arithmetic per piece (q the nibble, x the token in fp32 shared memory):
//   u = 1 + q/16 is built from the nibble by bit operations (exponent of 1.0 with q in the
//   top mantissa bits), d = sum u*x, so sum q*x = 16 (d - sum x) with sum x of the piece
//   precomputed once per block; the piece adds s * 16 (d - sx) + b * sx. fp32 throughout,
//   a warp-shuffle sum per row and one rounding to the output type.
//
// The token lives in shared memory as pieces of 32 floats padded to 36, so the eight lanes
// of each quarter-warp phase of a 128-bit shared load hit distinct banks.
#include "hsd_common.cuh"
#include "hsd_prefill.cuh"

namespace hsd {
// the tensor-core forms (csrc/hsd_qmma.cu) of the up and linear products
int qmma_moe_up(const void* x, int x_dtype, int64_t x_stride, const int32_t* sel, const uint32_t* uw,
                const void* us, const void* ub, int s_dtype, const uint32_t* suw, const void* sus, const void* sub,
                void* h, int h_dtype, int B, int D, int F, int FS, int topk, int E, cudaStream_t st);
int qmma_linear(const void* x, int x_dtype, int64_t x_stride, const uint32_t* w, const void* s, const void* b,
                int s_dtype, const void* resid, void* y, int y_dtype, int B, int in_f, int out_f, cudaStream_t st);
}  // namespace hsd

HSD_DEFINE_STATUS(up)

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kRowsPerWarp = 1;                         // one row per warp: many warps in flight
constexpr int kRowsPerBlock = kWarps * kRowsPerWarp;   // 16
constexpr int kPad = 36;                                // floats per 32-column piece in smem
constexpr int kMaxD = 8192;                             // longest reduction (8 pieces a lane)

enum Mode { kUp = 0, kDense = 1, kLinear = 2 };

struct UpParams {
  const void* x;
  int64_t x_stride;
  int x_dtype;
  const float* gains;     // dense form: [B, topk+1]
  const void* resid;      // linear form: [B, rows] in h_dtype, or null
  const int32_t* sel;
  const uint32_t* uw;
  const uint16_t* us;
  const uint16_t* ub;
  const uint32_t* suw;
  const uint16_t* sus;
  const uint16_t* sub;
  void* h;
  int h_dtype;
  int B, D, F, FS, topk, E;
  int tiles_routed, tiles_shared, tiles_per_b;
};
// Sizes per part: up form rows F / FS, reduction D; dense form rows D, reduction F / FS.

__device__ __forceinline__ float load_x(const void* x, int dtype, int64_t i) {
  switch (dtype) {
    case HSD_F32: return reinterpret_cast<const float*>(x)[i];
    case HSD_F16: return __half2float(reinterpret_cast<const __half*>(x)[i]);
    default: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(x)[i]);
  }
}

// 8 consecutive values x[i .. i+7] as fp32; vec: the address is 16-byte aligned
__device__ __forceinline__ void load8(const void* x, int dtype, int64_t i, bool vec, float* v) {
  if (vec && dtype != HSD_F32) {
    const uint4 r = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + i));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (dtype == HSD_BF16) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
      } else {
        v[2 * k] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[k] & 0xffffu)));
        v[2 * k + 1] = __half2float(__ushort_as_half(static_cast<uint16_t>(w[k] >> 16)));
      }
    }
  } else if (vec) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + i));
    const float4 b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(x) + i) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = load_x(x, dtype, i + k);
  }
}

__device__ __forceinline__ void store_h(void* h, int dtype, int64_t i, float v) {
  switch (dtype) {
    case HSD_F32: reinterpret_cast<float*>(h)[i] = v; break;
    case HSD_F16: reinterpret_cast<__half*>(h)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<__nv_bfloat16*>(h)[i] = __float2bfloat16_rn(v); break;
  }
}

// 1 + q/16 for nibble k of w: q moved to mantissa bits 19..22 under the exponent of 1.0.
template <int K>
__device__ __forceinline__ float nib_unit(uint32_t w) {
  constexpr int sh = 19 - 4 * K;
  uint32_t m;
  if constexpr (sh >= 0) m = w << sh;
  else m = w >> (-sh);
  return __uint_as_float((m & 0x00780000u) | 0x3F800000u);
}

// sum over the 8 nibbles of w of (1 + q/16) * x[0..7]
__device__ __forceinline__ float word_dot(uint32_t w, const float4 a, const float4 b, float acc) {
  acc = fmaf(nib_unit<0>(w), a.x, acc);
  acc = fmaf(nib_unit<1>(w), a.y, acc);
  acc = fmaf(nib_unit<2>(w), a.z, acc);
  acc = fmaf(nib_unit<3>(w), a.w, acc);
  acc = fmaf(nib_unit<4>(w), b.x, acc);
  acc = fmaf(nib_unit<5>(w), b.y, acc);
  acc = fmaf(nib_unit<6>(w), b.z, acc);
  acc = fmaf(nib_unit<7>(w), b.w, acc);
  return acc;
}

template <int MODE, typename ST, int MAXC>
__global__ void __launch_bounds__(kThreads) moe_qgemv_kernel(const UpParams p, int max_pieces) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  extern __shared__ __align__(16) float smem_f[];
  float* xs = smem_f;                               // [max_pieces][kPad]
  float* xsum = smem_f + max_pieces * kPad;         // [max_pieces]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bi = blockIdx.x / p.tiles_per_b;
  const int t = blockIdx.x % p.tiles_per_b;
  const int64_t hrow = static_cast<int64_t>(p.topk) * p.F + p.FS;   // h row length

  // which part, which weight rows, which reduction length
  const bool routed = t < p.topk * p.tiles_routed;
  const int part = routed ? t / p.tiles_routed : p.topk;
  const int tile = routed ? t % p.tiles_routed : t - p.topk * p.tiles_routed;
  const int red = MODE != kDense ? p.D : (routed ? p.F : p.FS);     // reduction length
  const int rows = MODE != kDense ? (routed ? p.F : p.FS) : p.D;
  const int NP = red / 32;          // pieces per row
  const int WR = red / 8;           // words per row
  const int GR = red / 64;          // groups per row
  const int64_t rows_per_expert = static_cast<int64_t>(rows);
  const uint32_t* W;
  const uint16_t* S;
  const uint16_t* Bz;
  bool bad = false;
  if (routed) {
    const int e = p.sel[bi * p.topk + part];
    if (e < 0 || e >= p.E) {
      bad = true;
      W = p.uw; S = p.us; Bz = p.ub;
    } else {
      W = p.uw + e * rows_per_expert * WR;
      S = p.us + e * rows_per_expert * GR;
      Bz = p.ub + e * rows_per_expert * GR;
    }
  } else {
    W = p.suw; S = p.sus; Bz = p.sub;
  }
  // output: up -> h[b, part*F + row] (bf16 etc.); dense -> partial rows [b, part, row] fp32
  const int64_t out0 = MODE == kUp      ? bi * hrow + static_cast<int64_t>(part) * p.F
                       : MODE == kDense ? (static_cast<int64_t>(bi) * (p.topk + 1) + part) * p.D
                                        : static_cast<int64_t>(bi) * p.FS;
  const int r0 = tile * kRowsPerBlock + warp * kRowsPerWarp;

  if (bad) {   // an expert id outside [0, E): zeros for the slot, recorded once per block
    if (tid == 0) hsd_flag_up(HSD_ERR_INDEX);
    if (lane < kRowsPerWarp && r0 + lane < rows) {
      if (MODE == kDense) reinterpret_cast<float*>(p.h)[out0 + r0 + lane] = 0.f;
      else store_h(p.h, p.h_dtype, out0 + r0 + lane, 0.f);
    }
    return;
  }

  // issue this warp's weight, scale and bias loads first: they do not depend on the token,
  // and none of them may wait behind another (each is a DRAM round trip)
  uint4 wv[kRowsPerWarp][MAXC];
  uint16_t sv[kRowsPerWarp][MAXC], bv[kRowsPerWarp][MAXC];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int row = min(r0 + r, rows - 1);
    const uint32_t* wr = W + static_cast<int64_t>(row) * WR;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int pc = lane + 32 * c;
      wv[r][c] = pc < NP ? hsd::ldg_nc_v4(wr + 4 * pc) : make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    const int row = min(r0 + r, rows - 1);
    const uint16_t* sr = S + static_cast<int64_t>(row) * GR;
    const uint16_t* br = Bz + static_cast<int64_t>(row) * GR;
#pragma unroll
    for (int c = 0; c < MAXC; ++c) {
      const int pc = lane + 32 * c;
      sv[r][c] = pc < NP ? __ldg(sr + (pc >> 1)) : static_cast<uint16_t>(0);
      bv[r][c] = pc < NP ? __ldg(br + (pc >> 1)) : static_cast<uint16_t>(0);
    }
  }

  // the input row, as padded 32-float pieces, and the sum of every piece: a thread loads a
  // quarter piece (8 values, one 16-byte load when the row is aligned), 4 adjacent lanes
  // sum a piece with two shuffles
  const int64_t xb = static_cast<int64_t>(bi) * p.x_stride + (MODE != kDense ? 0 : static_cast<int64_t>(part) * p.F);
  const int esz = p.x_dtype == HSD_F32 ? 4 : 2;
  const bool vec = (reinterpret_cast<uintptr_t>(p.x) + static_cast<uintptr_t>(xb) * esz) % 16 == 0;
  const int nq = red / 8;
  for (int q0 = 0; q0 < nq; q0 += kThreads) {
    const int q = q0 + tid;
    float v[8];
    if (q < nq) load8(p.x, p.x_dtype, xb + 8 * q, vec, v);
    else
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    float sq = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    sq += __shfl_xor_sync(0xffffffffu, sq, 1);
    sq += __shfl_xor_sync(0xffffffffu, sq, 2);
    if (q < nq) {
      float4* dst = reinterpret_cast<float4*>(xs + (q >> 2) * kPad + (q & 3) * 8);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
      if ((q & 3) == 0) xsum[q >> 2] = sq;
    }
  }
  __syncthreads();

  // a piece of the token is read from shared memory once and applied to the warp's rows;
  // each row still accumulates its pieces in ascending order
  float accr[kRowsPerWarp];
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) accr[r] = 0.f;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int pc = lane + 32 * c;
    if (pc < NP) {
      const float4* xp = reinterpret_cast<const float4*>(xs + pc * kPad);
      float4 xv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[i] = xp[i];
      const float sx = xsum[pc];
#pragma unroll
      for (int r = 0; r < kRowsPerWarp; ++r) {
        float d = 0.f;
        d = word_dot(wv[r][c].x, xv[0], xv[1], d);
        d = word_dot(wv[r][c].y, xv[2], xv[3], d);
        d = word_dot(wv[r][c].z, xv[4], xv[5], d);
        d = word_dot(wv[r][c].w, xv[6], xv[7], d);
        const float sc = hsd::bits16_to_f32<ST>(sv[r][c]);
        const float bc = hsd::bits16_to_f32<ST>(bv[r][c]);
        accr[r] = fmaf(sc * 16.f, d - sx, fmaf(bc, sx, accr[r]));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kRowsPerWarp; ++r) {
    float acc = accr[r];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0 && r0 + r < rows) {
      if (MODE == kUp) {
        const float v = fmaxf(acc, 0.f);
        store_h(p.h, p.h_dtype, out0 + r0 + r, v * v);
      } else if (MODE == kDense) {
        reinterpret_cast<float*>(p.h)[out0 + r0 + r] = p.gains[bi * (p.topk + 1) + part] * acc;
      } else {
        const float rv = p.resid ? load_x(p.resid, p.h_dtype, out0 + r0 + r) : 0.f;
        store_h(p.h, p.h_dtype, out0 + r0 + r, rv + acc);
      }
    }
  }
}

template <int MODE, typename ST, int MAXC>
int launch_c(const UpParams& p, int max_pieces, int grid, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(max_pieces) * (kPad + 1) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(moe_qgemv_kernel<MODE, ST, MAXC>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return hsd::check_cuda(e, "qgemv smem attribute");
  }
  hsd::launch_pdl(moe_qgemv_kernel<MODE, ST, MAXC>, dim3(grid), dim3(kThreads), smem, st, p, max_pieces);
  return HSD_OK;
}

template <int MODE, typename ST>
int launch_qgemv(const UpParams& p, int max_red, int grid, cudaStream_t st, const char* who) {
  const int pieces = max_red / 32;
  int rc;
  switch ((pieces + 31) / 32) {
    case 1: rc = launch_c<MODE, ST, 1>(p, pieces, grid, st); break;
    case 2: rc = launch_c<MODE, ST, 2>(p, pieces, grid, st); break;
    case 3: rc = launch_c<MODE, ST, 3>(p, pieces, grid, st); break;
    case 4: rc = launch_c<MODE, ST, 4>(p, pieces, grid, st); break;
    case 5: case 6: rc = launch_c<MODE, ST, 6>(p, pieces, grid, st); break;
    default: rc = launch_c<MODE, ST, 8>(p, pieces, grid, st); break;
  }
  if (rc != HSD_OK) return rc;
  return hsd::check_launch(who);
}

}  // namespace

extern "C" int hsd_moe_up_decode(const void* x, int x_dtype, int64_t x_stride, const int32_t* sel,
                                 const uint32_t* uw, const void* us, const void* ub, int s_dtype,
                                 const uint32_t* suw, const void* sus, const void* sub, void* h,
                                 int h_dtype, int B, int D, int F, int FS, int topk, int E,
                                 void* stream) {
  if (B < 0 || topk < 0 || F < 0 || FS < 0 || E < 0)
    return hsd::set_error(HSD_ERR_ARG, "hsd_moe_up_decode: negative size");
  if (B == 0 || topk * F + FS == 0) return HSD_OK;
  if (D <= 0 || D % 64 != 0 || D > kMaxD)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_moe_up_decode: need D %% 64 == 0 and D <= %d (D=%d)", kMaxD, D);
  if (x_dtype < HSD_F32 || x_dtype > HSD_BF16 || h_dtype < HSD_F32 || h_dtype > HSD_BF16)
    return hsd::set_error(HSD_ERR_DTYPE, "hsd_moe_up_decode: x / h dtype codes %d / %d", x_dtype, h_dtype);
  if (s_dtype != HSD_F16 && s_dtype != HSD_BF16)
    return hsd::set_error(HSD_ERR_DTYPE, "hsd_moe_up_decode: scales must be f16 or bf16 (code %d)", s_dtype);
  if (!x || !h || x_stride < D) return hsd::set_error(HSD_ERR_ARG, "hsd_moe_up_decode: null x / h or x_stride < D");
  if (topk > 0 && (!sel || !uw || !us || !ub || F <= 0 || E <= 0))
    return hsd::set_error(HSD_ERR_ARG, "hsd_moe_up_decode: routed part needs sel, uw, us, ub, F > 0, E > 0");
  if (FS > 0 && (!suw || !sus || !sub))
    return hsd::set_error(HSD_ERR_ARG, "hsd_moe_up_decode: shared part needs suw, sus, sub");
  if ((topk > 0 && !hsd::aligned(uw, 16)) || (FS > 0 && !hsd::aligned(suw, 16)))
    return hsd::set_error(HSD_ERR_ALIGN, "hsd_moe_up_decode: packed weights must be 16-byte aligned");
  return hsd::qmma_moe_up(x, x_dtype, x_stride, sel, uw, us, ub, s_dtype, suw, sus, sub, h, h_dtype, B, D, F, FS,
                          topk, E, hsd::as_stream(stream));
}

extern "C" int hsd_dense_down_decode(const void* h, int h_dtype, const int32_t* sel, const float* gains,
                                     const uint32_t* w, const void* s, const void* b, int s_dtype,
                                     const uint32_t* sw, const void* ss, const void* sb, const void* resid,
                                     void* y, int y_dtype, float* part, int B, int D, int F, int FS, int topk,
                                     int E, void* stream) {
  const char* who = "hsd_dense_down_decode";
  if (B < 0 || topk < 0 || F < 0 || FS < 0 || E < 0) return hsd::set_error(HSD_ERR_ARG, "%s: negative size", who);
  if (B == 0) return HSD_OK;
  if (D <= 0 || D % 32 != 0 || F % 64 != 0 || FS % 64 != 0 || F > kMaxD || FS > kMaxD || topk * F + FS == 0)
    return hsd::set_error(HSD_ERR_SHAPE, "%s: need D %% 32 == 0, F and FS multiples of 64 and <= %d", who, kMaxD);
  if (h_dtype < HSD_F32 || h_dtype > HSD_BF16 || y_dtype < HSD_F32 || y_dtype > HSD_BF16)
    return hsd::set_error(HSD_ERR_DTYPE, "%s: h / y dtype codes %d / %d", who, h_dtype, y_dtype);
  if (s_dtype != HSD_F16 && s_dtype != HSD_BF16)
    return hsd::set_error(HSD_ERR_DTYPE, "%s: scales must be f16 or bf16 (code %d)", who, s_dtype);
  if (!h || !gains || !y || !part) return hsd::set_error(HSD_ERR_ARG, "%s: null h / gains / y / part", who);
  if (topk > 0 && (!sel || !w || !s || !b || F <= 0 || E <= 0))
    return hsd::set_error(HSD_ERR_ARG, "%s: routed part needs sel, w, s, b, F > 0, E > 0", who);
  if (FS > 0 && (!sw || !ss || !sb)) return hsd::set_error(HSD_ERR_ARG, "%s: shared part needs sw, ss, sb", who);
  if ((topk > 0 && !hsd::aligned(w, 16)) || (FS > 0 && !hsd::aligned(sw, 16)))
    return hsd::set_error(HSD_ERR_ALIGN, "%s: packed weights must be 16-byte aligned", who);
  UpParams p;
  p.x = h; p.x_stride = static_cast<int64_t>(topk) * F + FS; p.x_dtype = h_dtype; p.sel = sel; p.gains = gains;
  p.resid = nullptr;
  p.uw = w; p.us = static_cast<const uint16_t*>(s); p.ub = static_cast<const uint16_t*>(b);
  p.suw = sw; p.sus = static_cast<const uint16_t*>(ss); p.sub = static_cast<const uint16_t*>(sb);
  p.h = part; p.h_dtype = HSD_F32;
  p.B = B; p.D = D; p.F = F; p.FS = FS; p.topk = topk; p.E = E;
  const int tiles = (D + kRowsPerBlock - 1) / kRowsPerBlock;
  p.tiles_routed = topk > 0 ? tiles : 0;
  p.tiles_shared = FS > 0 ? tiles : 0;
  p.tiles_per_b = topk * p.tiles_routed + p.tiles_shared;
  const int64_t grid = static_cast<int64_t>(B) * p.tiles_per_b;
  if (grid > 0x7fffffff) return hsd::set_error(HSD_ERR_SHAPE, "%s: grid too large", who);
  cudaStream_t st = hsd::as_stream(stream);
  const int max_red = F > FS ? F : FS;
  int rc = s_dtype == HSD_BF16 ? launch_qgemv<kDense, __nv_bfloat16>(p, max_red, static_cast<int>(grid), st, who)
                               : launch_qgemv<kDense, __half>(p, max_red, static_cast<int>(grid), st, who);
  if (rc != HSD_OK) return rc;
  return hsd::launch_reduce(part, resid, y, y_dtype, B, D, topk, topk + (FS > 0 ? 1 : 0), st);
}

extern "C" int hsd_qlinear_decode(const void* x, int x_dtype, int64_t x_stride, const uint32_t* w, const void* s,
                                  const void* b, int s_dtype, const void* resid, void* y, int y_dtype, int B,
                                  int in_f, int out_f, void* stream) {
  const char* who = "hsd_qlinear_decode";
  if (B < 0 || in_f < 0 || out_f < 0) return hsd::set_error(HSD_ERR_ARG, "%s: negative size", who);
  if (B == 0 || out_f == 0) return HSD_OK;
  if (in_f <= 0 || in_f % 64 != 0 || in_f > kMaxD)
    return hsd::set_error(HSD_ERR_SHAPE, "%s: need in_f %% 64 == 0 and in_f <= %d (in_f=%d)", who, kMaxD, in_f);
  if (x_dtype < HSD_F32 || x_dtype > HSD_BF16 || y_dtype < HSD_F32 || y_dtype > HSD_BF16)
    return hsd::set_error(HSD_ERR_DTYPE, "%s: x / y dtype codes %d / %d", who, x_dtype, y_dtype);
  if (s_dtype != HSD_F16 && s_dtype != HSD_BF16)
    return hsd::set_error(HSD_ERR_DTYPE, "%s: scales must be f16 or bf16 (code %d)", who, s_dtype);
  if (!x || !w || !s || !b || !y || x_stride < in_f)
    return hsd::set_error(HSD_ERR_ARG, "%s: null pointer or x_stride < in_f", who);
  if (!hsd::aligned(w, 16)) return hsd::set_error(HSD_ERR_ALIGN, "%s: packed weights must be 16-byte aligned", who);
  return hsd::qmma_linear(x, x_dtype, x_stride, w, s, b, s_dtype, resid, y, y_dtype, B, in_f, out_f,
                          hsd::as_stream(stream));
}
