// The small per-row operators of a decode step around the hot path, fused so a captured
// step is a few launches per layer instead of a dozen elementwise ones:
//
//   rms_norm        y = w * cast(x * rsqrt(mean(x^2) + eps))  (NemotronH's RMSNorm: the
//                   normalised row is rounded to the row's dtype before the weight multiply,
//                   mlx-lm nemotron_h / transformers NemotronHRMSNorm)
//   gated_rms_norm  g = y * silu(gate); per group of `group` channels
//                   out = w * cast(g * rsqrt(mean(g^2) + eps))  (the Mamba-2 mixer's gated norm)
//   router_topk     the MoE router of hsd/model.py:115 (mix.gate): logits = x . R_e in fp32,
//                   scores = sigmoid(logits), the top-k experts by score (ties -> lower id),
//                   gains = scores / sum(top-k scores), and gain 1 for the shared expert.
//                   One block per (expert, row); the last block to finish (a ticket
//                   counter in caller memory, taken with one atomic, no waiting) selects the
//                   top k and resets the ticket for the next call.
//
// One block per row for the norms; fp32 arithmetic, warp-shuffle then shared-memory sums.
#include "hsd_common.cuh"

HSD_DEFINE_STATUS(norm)

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case HSD_F32: return reinterpret_cast<const float*>(p)[i];
    case HSD_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    default: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  }
}

// round v to `dtype` and back (the cast before the weight multiply)
__device__ __forceinline__ float round_to(float v, int dtype) {
  switch (dtype) {
    case HSD_F32: return v;
    case HSD_F16: return __half2float(__float2half_rn(v));
    default: return __bfloat162float(__float2bfloat16_rn(v));
  }
}

__device__ __forceinline__ void store_any(void* p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case HSD_F32: reinterpret_cast<float*>(p)[i] = v; break;
    case HSD_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();                       // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  return t;
}

__global__ void __launch_bounds__(kThreads) rms_norm_kernel(const void* x, int x_dtype, int64_t x_stride,
                                                             const void* w, int w_dtype, void* y, int y_dtype,
                                                             int D, float eps) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  __shared__ float red[kThreads / 32];
  const int64_t r = blockIdx.x;
  const int64_t xo = r * x_stride;
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += kThreads) {
    const float v = load_any(x, x_dtype, xo + i);
    ss = fmaf(v, v, ss);
  }
  const float rs = rsqrtf(block_sum(ss, red) / D + eps);
  for (int i = threadIdx.x; i < D; i += kThreads) {
    const float n = round_to(load_any(x, x_dtype, xo + i) * rs, x_dtype);
    store_any(y, y_dtype, r * D + i, round_to(load_any(w, w_dtype, i) * n, y_dtype));
  }
}

// bf16 rows, D % 8 == 0, 16-byte aligned: each thread keeps its NV 8-value pieces in
// registers, so the row is read once (the same arithmetic as rms_norm_kernel).
template <int NV>
__global__ void __launch_bounds__(kThreads) rms_norm_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride,
                                                                  const __nv_bfloat16* __restrict__ w,
                                                                  __nv_bfloat16* __restrict__ y, int D, float eps) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  __shared__ float red[kThreads / 32];
  const int64_t r = blockIdx.x;
  const int nq = D / 8;
  uint4 xv[NV];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int q = threadIdx.x + k * kThreads;
    xv[k] = q < nq ? __ldg(reinterpret_cast<const uint4*>(x + r * x_stride) + q) : make_uint4(0, 0, 0, 0);
    const uint32_t wd[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = __uint_as_float(wd[i] << 16), b = __uint_as_float(wd[i] & 0xffff0000u);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
  }
  const float rs = rsqrtf(block_sum(ss, red) / D + eps);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int q = threadIdx.x + k * kThreads;
    if (q >= nq) continue;
    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + q);
    const uint32_t xd[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t od[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float n0 = round_to(__uint_as_float(xd[i] << 16) * rs, HSD_BF16);
      const float n1 = round_to(__uint_as_float(xd[i] & 0xffff0000u) * rs, HSD_BF16);
      const __nv_bfloat16 o0 = __float2bfloat16_rn(__uint_as_float(wd[i] << 16) * n0);
      const __nv_bfloat16 o1 = __float2bfloat16_rn(__uint_as_float(wd[i] & 0xffff0000u) * n1);
      od[i] = static_cast<uint32_t>(__bfloat16_as_ushort(o0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(o1)) << 16);
    }
    reinterpret_cast<uint4*>(y + r * D)[q] = make_uint4(od[0], od[1], od[2], od[3]);
  }
}

__global__ void __launch_bounds__(kThreads) gated_rms_norm_kernel(const void* yv, int y_dtype, int64_t y_stride,
                                                                   const void* gate, int g_dtype, int64_t g_stride,
                                                                   const void* w, int w_dtype, void* out,
                                                                   int out_dtype, int I, int group, float eps) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  // one block per (row, group): blockIdx.x = row * (I / group) + group index
  __shared__ float red[kThreads / 32];
  const int ng = I / group;
  const int64_t r = blockIdx.x / ng;
  const int c0 = (blockIdx.x % ng) * group;
  float ss = 0.f;
  for (int i = threadIdx.x; i < group; i += kThreads) {
    const float gt = load_any(gate, g_dtype, r * g_stride + c0 + i);
    const float v = load_any(yv, y_dtype, r * y_stride + c0 + i) * (gt / (1.f + expf(-gt)));
    ss = fmaf(v, v, ss);
  }
  const float rs = rsqrtf(block_sum(ss, red) / group + eps);
  for (int i = threadIdx.x; i < group; i += kThreads) {
    const float gt = load_any(gate, g_dtype, r * g_stride + c0 + i);
    const float v = load_any(yv, y_dtype, r * y_stride + c0 + i) * (gt / (1.f + expf(-gt)));
    const float n = round_to(v * rs, out_dtype);
    store_any(out, out_dtype, r * I + c0 + i, round_to(load_any(w, w_dtype, c0 + i) * n, out_dtype));
  }
}

// ---- router: logits, sigmoid, top-k, normalised gains ------------------------------
constexpr int kRouterThreads = 128;      // one block per (expert, row)
constexpr int kRouterWarps = kRouterThreads / 32;
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopk = 16;

// KP: scores a lane holds in the top-k selection (32 * KP >= E), so the selection's loops
// cover only the experts there are.
template <int KP>
__global__ void __launch_bounds__(kRouterThreads) router_topk_kernel(const void* x, int x_dtype, int64_t x_stride,
                                                                      const float* __restrict__ R, int B, int D,
                                                                      int E, int topk, float* scores,
                                                                      unsigned int* ticket, int32_t* sel,
                                                                      float* gains) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  // grid: (E, B); scores [B, E] fp32 scratch
  __shared__ float red[kRouterWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e = blockIdx.x, b = blockIdx.y;
  {
    const float* re = R + static_cast<int64_t>(e) * D;
    const int64_t xo = static_cast<int64_t>(b) * x_stride;
    float acc = 0.f;
    const bool vec = x_dtype == HSD_BF16 && D % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(static_cast<const uint16_t*>(x) + xo) % 8) == 0 &&
                     (reinterpret_cast<uintptr_t>(re) % 16) == 0;
    if (vec) {                           // 4 weights (16 bytes) and 4 bf16 inputs (8 bytes) a load
      const float4* r4 = reinterpret_cast<const float4*>(re);
      const uint2* x4 = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + xo);
#pragma unroll 4
      for (int c = threadIdx.x; c < D / 4; c += kRouterThreads) {
        const float4 rv = __ldg(r4 + c);
        const uint2 xv = __ldg(x4 + c);
        acc = fmaf(__uint_as_float(xv.x << 16), rv.x, acc);
        acc = fmaf(__uint_as_float(xv.x & 0xffff0000u), rv.y, acc);
        acc = fmaf(__uint_as_float(xv.y << 16), rv.z, acc);
        acc = fmaf(__uint_as_float(xv.y & 0xffff0000u), rv.w, acc);
      }
    } else {
      for (int i = threadIdx.x; i < D; i += kRouterThreads) acc = fmaf(load_any(x, x_dtype, xo + i), re[i], acc);
    }
    const float t = block_sum(acc, red);
    if (threadIdx.x == 0) scores[static_cast<int64_t>(b) * E + e] = 1.f / (1.f + expf(-t));
  }
  // the last block of the whole grid selects the top k of every row
  __shared__ bool last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned total = gridDim.x * gridDim.y;
    last = atomicAdd(ticket, 1u) == total - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (threadIdx.x == 0) *ticket = 0u;
  // one warp per row: the row's scores into registers once (KP per lane), then k rounds of a
  // warp arg-max over them (ties -> lower id)
  constexpr int kPer = KP;
  for (int row = warp; row < B; row += kRouterWarps) {
    const volatile float* sc = scores + static_cast<int64_t>(row) * E;
    float v[kPer];
#pragma unroll
    for (int t = 0; t < kPer; ++t) {
      const int i = lane + 32 * t;
      v[t] = i < E ? sc[i] : -INFINITY;
    }
    float total = 0.f, chosen = 0.f;
    for (int k = 0; k < topk; ++k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const int i = lane + 32 * t;
        if (v[t] > bv || (v[t] == bv && i < bi)) { bv = v[t]; bi = i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      // the owner lane retires the chosen entry; lane k keeps the k-th choice
#pragma unroll
      for (int t = 0; t < kPer; ++t)
        if (lane + 32 * t == bi) v[t] = -INFINITY;
      if (lane == k) chosen = bv;
      if (lane == 0) sel[static_cast<int64_t>(row) * topk + k] = bi;
      total += bv;
    }
    if (lane < topk) gains[static_cast<int64_t>(row) * (topk + 1) + lane] = chosen / (total + 1e-20f);
    if (lane == 0) gains[static_cast<int64_t>(row) * (topk + 1) + topk] = 1.f;
  }
}

bool dtype_ok(int d) { return d >= HSD_F32 && d <= HSD_BF16; }

}  // namespace

extern "C" int hsd_rms_norm(const void* x, int x_dtype, int64_t x_stride, const void* w, int w_dtype, void* y,
                            int y_dtype, int B, int D, float eps, void* stream) {
  if (B < 0 || D < 1) return hsd::set_error(HSD_ERR_SHAPE, "hsd_rms_norm: need B >= 0, D >= 1");
  if (B == 0) return HSD_OK;
  if (!x || !w || !y || x_stride < D) return hsd::set_error(HSD_ERR_ARG, "hsd_rms_norm: null pointer or x_stride < D");
  if (!dtype_ok(x_dtype) || !dtype_ok(w_dtype) || !dtype_ok(y_dtype))
    return hsd::set_error(HSD_ERR_DTYPE, "hsd_rms_norm: dtype codes %d %d %d", x_dtype, w_dtype, y_dtype);
  cudaStream_t st = hsd::as_stream(stream);
  const int nv = (D / 8 + kThreads - 1) / kThreads;
  if (x_dtype == HSD_BF16 && w_dtype == HSD_BF16 && y_dtype == HSD_BF16 && D % 8 == 0 && nv <= 4 &&
      x_stride % 8 == 0 && hsd::aligned(x, 16) && hsd::aligned(w, 16) && hsd::aligned(y, 16)) {
    const auto* xb = static_cast<const __nv_bfloat16*>(x);
    const auto* wb = static_cast<const __nv_bfloat16*>(w);
    auto* yb = static_cast<__nv_bfloat16*>(y);
    switch (nv) {
      case 1: hsd::launch_pdl(rms_norm_bf16_kernel<1>, dim3(B), dim3(kThreads), 0, st, xb, x_stride, wb, yb, D, eps); break;
      case 2: hsd::launch_pdl(rms_norm_bf16_kernel<2>, dim3(B), dim3(kThreads), 0, st, xb, x_stride, wb, yb, D, eps); break;
      case 3: hsd::launch_pdl(rms_norm_bf16_kernel<3>, dim3(B), dim3(kThreads), 0, st, xb, x_stride, wb, yb, D, eps); break;
      default: hsd::launch_pdl(rms_norm_bf16_kernel<4>, dim3(B), dim3(kThreads), 0, st, xb, x_stride, wb, yb, D, eps); break;
    }
  } else {
    hsd::launch_pdl(rms_norm_kernel, dim3(B), dim3(kThreads), 0, st, x, x_dtype, x_stride, w, w_dtype, y, y_dtype, D, eps);
  }
  return hsd::check_launch("hsd_rms_norm");
}

extern "C" int hsd_gated_rms_norm(const void* y, int y_dtype, int64_t y_stride, const void* gate, int g_dtype,
                                  int64_t g_stride, const void* w, int w_dtype, void* out, int out_dtype, int B,
                                  int I, int group, float eps, void* stream) {
  if (B < 0 || I < 1 || group < 1 || I % group != 0)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_gated_rms_norm: need I %% group == 0");
  if (B == 0) return HSD_OK;
  if (!y || !gate || !w || !out || y_stride < I || g_stride < I)
    return hsd::set_error(HSD_ERR_ARG, "hsd_gated_rms_norm: null pointer or stride < I");
  if (!dtype_ok(y_dtype) || !dtype_ok(g_dtype) || !dtype_ok(w_dtype) || !dtype_ok(out_dtype))
    return hsd::set_error(HSD_ERR_DTYPE, "hsd_gated_rms_norm: bad dtype code");
  const int64_t grid = static_cast<int64_t>(B) * (I / group);
  if (grid > 0x7fffffff) return hsd::set_error(HSD_ERR_SHAPE, "hsd_gated_rms_norm: grid too large");
  hsd::launch_pdl(gated_rms_norm_kernel, dim3(static_cast<unsigned>(grid)), dim3(kThreads), 0, hsd::as_stream(stream),
      y, y_dtype, y_stride, gate, g_dtype, g_stride, w, w_dtype, out, out_dtype, I, group, eps);
  return hsd::check_launch("hsd_gated_rms_norm");
}

extern "C" int hsd_router_topk(const void* x, int x_dtype, int64_t x_stride, const float* R, int B, int D, int E,
                               int topk, float* scores, unsigned int* ticket, int32_t* sel, float* gains,
                               void* stream) {
  if (B < 0 || D < 1 || E < 1 || E > kMaxExperts || topk < 1 || topk > kMaxTopk || topk > E || B > 65535)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_router_topk: need 1 <= topk <= min(E, %d), E <= %d, B <= 65535",
                          kMaxTopk, kMaxExperts);
  if (B == 0) return HSD_OK;
  if (!x || !R || !scores || !ticket || !sel || !gains || x_stride < D)
    return hsd::set_error(HSD_ERR_ARG, "hsd_router_topk: null pointer or x_stride < D");
  if (!dtype_ok(x_dtype)) return hsd::set_error(HSD_ERR_DTYPE, "hsd_router_topk: x dtype code %d", x_dtype);
  dim3 grid(E, B);
  cudaStream_t st = hsd::as_stream(stream);
  if (E <= 128)
    hsd::launch_pdl(router_topk_kernel<4>, grid, dim3(kRouterThreads), 0, st, x, x_dtype, x_stride, R, B, D, E, topk,
                    scores, ticket, sel, gains);
  else if (E <= 256)
    hsd::launch_pdl(router_topk_kernel<8>, grid, dim3(kRouterThreads), 0, st, x, x_dtype, x_stride, R, B, D, E, topk,
                    scores, ticket, sel, gains);
  else
    hsd::launch_pdl(router_topk_kernel<kMaxExperts / 32>, grid, dim3(kRouterThreads), 0, st, x, x_dtype, x_stride, R,
                    B, D, E, topk, scores, ticket, sel, gains);
  return hsd::check_launch("hsd_router_topk");
}
