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
//                   One warp per expert over all blocks; the last block to finish (a ticket
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

__global__ void __launch_bounds__(kThreads) gated_rms_norm_kernel(const void* yv, int y_dtype, int64_t y_stride,
                                                                   const void* gate, int g_dtype, int64_t g_stride,
                                                                   const void* w, int w_dtype, void* out,
                                                                   int out_dtype, int I, int group, float eps) {
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
constexpr int kRouterWarps = 8;          // experts per block
constexpr int kMaxExperts = 1024;
constexpr int kMaxTopk = 16;

__global__ void __launch_bounds__(kRouterWarps * 32) router_topk_kernel(const void* x, int x_dtype, int64_t x_stride,
                                                                         const float* __restrict__ R, int B, int D,
                                                                         int E, int topk, float* scores,
                                                                         unsigned int* ticket, int32_t* sel,
                                                                         float* gains) {
  // grid: (ceil(E / kRouterWarps), B); scores [B, E] fp32 scratch
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.y;
  const int e = blockIdx.x * kRouterWarps + warp;
  if (e < E) {
    const float* re = R + static_cast<int64_t>(e) * D;
    const int64_t xo = static_cast<int64_t>(b) * x_stride;
    float acc = 0.f;
    for (int i = lane; i < D; i += 32) acc = fmaf(load_any(x, x_dtype, xo + i), re[i], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) scores[static_cast<int64_t>(b) * E + e] = 1.f / (1.f + expf(-acc));
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
  // one warp per row: k rounds of a warp arg-max over the row's scores (ties -> lower id)
  for (int row = warp; row < B; row += kRouterWarps) {
    const volatile float* sc = scores + static_cast<int64_t>(row) * E;
    float chosen_val[kMaxTopk];
    int chosen_id[kMaxTopk];
    float total = 0.f;
    for (int k = 0; k < topk; ++k) {
      float bv = -1.f;
      int bi = 0x7fffffff;
      for (int i = lane; i < E; i += 32) {
        bool taken = false;
        for (int j = 0; j < k; ++j) taken |= (chosen_id[j] == i);
        const float v = sc[i];
        if (!taken && (v > bv || (v == bv && i < bi))) { bv = v; bi = i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      chosen_val[k] = bv;
      chosen_id[k] = bi;
      total += bv;
    }
    if (lane == 0) {
      for (int k = 0; k < topk; ++k) {
        sel[static_cast<int64_t>(row) * topk + k] = chosen_id[k];
        gains[static_cast<int64_t>(row) * (topk + 1) + k] = chosen_val[k] / (total + 1e-20f);
      }
      gains[static_cast<int64_t>(row) * (topk + 1) + topk] = 1.f;
    }
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
  rms_norm_kernel<<<B, kThreads, 0, hsd::as_stream(stream)>>>(x, x_dtype, x_stride, w, w_dtype, y, y_dtype, D, eps);
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
  gated_rms_norm_kernel<<<static_cast<unsigned>(grid), kThreads, 0, hsd::as_stream(stream)>>>(
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
  dim3 grid((E + kRouterWarps - 1) / kRouterWarps, B);
  router_topk_kernel<<<grid, kRouterWarps * 32, 0, hsd::as_stream(stream)>>>(x, x_dtype, x_stride, R, B, D, E, topk,
                                                                             scores, ticket, sel, gains);
  return hsd::check_launch("hsd_router_topk");
}
