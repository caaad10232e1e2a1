// Mamba-2 multi-row verify with per-row checkpointed state, and the rollback to an accepted
// prefix (hsd/mamba.py:19-56 of the reference, which records the verify's inputs and re-runs
// mlx-lm's ssm_update over the kept rows; here every row's state is written once during the
// verify, so a rollback is a selection and never a recomputation).
//
// conv_verify  one thread per channel with a rolling 4-row register window: the window
//              [conv_state; conv_in] (K-1+L rows) is copied to `padded` and out[t] =
//              silu(bias + sum_j w[c, j] * padded[t + j]) in fp32. After keeping n rows the
//              conv state is padded[n : n+K-1].
// ssm_verify   one warp per (head h, channel p); lane l holds state[h, p, l*NPL .. +NPL) in
//              registers. Rows one after another, exactly as single steps would run them:
//                dt_t = clamp(softplus(dt[t,h] + dt_bias[h]), dt_min, dt_max)
//                state = state * exp(dt_t * A_h) + (dt_t * x[t,h,p]) * B[t, g(h), :]
//                y[t,h,p] = sum_n state * C[t, g(h), :] + D_h * x[t,h,p]   (warp reduction)
//              and after every row the warp stores its state slice to states[t] (coalesced);
//              with last_only (prefill, no rollback) only the final state, to states[0].
//              A verify of L rows and L single steps run the same instructions per row, so
//              the state after row n of a verify is bit-identical to n single steps.
//
// The *_step entry points are the same kernels on resident buffers, for decode loops that
// replay a captured CUDA graph: the conv window and the SSM state are read from the previous
// call's own output rows, selected by a device-side accepted-row count n_keep (the window
// padded[n_keep .. n_keep+K-2], the state states[n_keep-1]), and the new rows are written
// over the same buffers. Each thread (conv) or lane (ssm) reads its whole slice before it
// writes any of it, and only its own slice, so the in-place update needs no barrier. A
// rollback is then one integer written on the device.
#include <algorithm>

#include "hsd_common.cuh"

HSD_DEFINE_STATUS(mamba)

namespace {

// The accepted-row count of a resident-buffer call: *n_keep, or 1 (with HSD_ERR_INDEX in the
// status word) when it lies outside 1..rows.
__device__ __forceinline__ int read_keep(const int* n_keep, int rows) {
  const int k = *n_keep;
  if (k < 1 || k > rows) {
    if (threadIdx.x == 0) atomicCAS(&hsd_status_word_mamba, 0, HSD_ERR_INDEX);
    return 1;
  }
  return k;
}

template <typename T>
__device__ __forceinline__ float ld(const void* p, int64_t i) {
  return hsd::to_f32<T>(reinterpret_cast<const T*>(p)[i]);
}

// Four consecutive values at element index i (4-element aligned) as fp32, one vector load.
template <typename T>
__device__ __forceinline__ void ld4(const void* p, int64_t i, float* out) {
  if constexpr (sizeof(T) == 4) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
    out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
  } else {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const T*>(p) + i));
    out[0] = hsd::bits16_to_f32<T>(static_cast<uint16_t>(v.x & 0xffffu));
    out[1] = hsd::bits16_to_f32<T>(static_cast<uint16_t>(v.x >> 16));
    out[2] = hsd::bits16_to_f32<T>(static_cast<uint16_t>(v.y & 0xffffu));
    out[3] = hsd::bits16_to_f32<T>(static_cast<uint16_t>(v.y >> 16));
  }
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + expf(-x)); }
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }

template <typename TI, typename TW, typename TO>
__global__ void __launch_bounds__(256) conv_verify_kernel(const void* conv_in, int64_t in_stride,
                                                          const void* conv_state, const void* w,
                                                          const void* bias, void* out, void* padded, int L,
                                                          int C, const int* n_keep, int rows) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  constexpr int K = 4;                             // the model's conv kernel (checked on the host)
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c >= C) return;
  if (n_keep)                                      // resident form: the window is padded[n_keep ..]
    conv_state = static_cast<const TI*>(padded) + static_cast<int64_t>(read_keep(n_keep, rows)) * C;
  float win[K];                                    // rolling window: rows t .. t+K-1 of padded
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = conv_state ? ld<TI>(conv_state, static_cast<int64_t>(j) * C + c) : 0.f;
#pragma unroll
  for (int j = 0; j < K - 1; ++j)
    reinterpret_cast<TI*>(padded)[static_cast<int64_t>(j) * C + c] = hsd::from_f32<TI>(win[j]);
  const float b = bias ? ld<TW>(bias, c) : 0.f;
  float wk[K];
#pragma unroll
  for (int j = 0; j < K; ++j) wk[j] = ld<TW>(w, static_cast<int64_t>(c) * K + j);
  for (int t = 0; t < L; ++t) {
    win[K - 1] = ld<TI>(conv_in, static_cast<int64_t>(t) * in_stride + c);
    reinterpret_cast<TI*>(padded)[static_cast<int64_t>(K - 1 + t) * C + c] = hsd::from_f32<TI>(win[K - 1]);
    float a = b;
#pragma unroll
    for (int j = 0; j < K; ++j) a = fmaf(wk[j], win[j], a);
    reinterpret_cast<TO*>(out)[static_cast<int64_t>(t) * C + c] = hsd::from_f32<TO>(silu_f(a));
#pragma unroll
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
}

template <typename TX, typename TD, typename TY, int NPL>
__global__ void __launch_bounds__(256) ssm_verify_kernel(const void* xbc, int64_t xbc_stride, const void* dt,
                                                         int64_t dt_stride, const float* __restrict__ A_log,
                                                         const float* __restrict__ Dp,
                                                         const float* __restrict__ dt_bias, float dt_min,
                                                         float dt_max, const float* state0, float* states,
                                                         void* y, int L, int H, int P, int G, int N, int last_only,
                                                         const int* n_keep, int rows) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  const int warp_g = (blockIdx.x * 256 + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_g >= H * P) return;
  const int h = warp_g / P, p = warp_g - h * P;
  const int g = h / (H / G);
  const int I = H * P;
  const int64_t sbase = (static_cast<int64_t>(h) * P + p) * N + lane * NPL;   // this lane's slice
  if (n_keep) state0 = states + static_cast<int64_t>(read_keep(n_keep, rows) - 1) * H * P * N;
  float st[NPL];
  if constexpr (NPL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < NPL; i += 4) {
      const float4 v = state0 ? *reinterpret_cast<const float4*>(state0 + sbase + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      st[i] = v.x; st[i + 1] = v.y; st[i + 2] = v.z; st[i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NPL; ++i) st[i] = state0 ? state0[sbase + i] : 0.f;
  }
  const float A = -expf(A_log[h]);
  const float dbias = dt_bias[h], Dh = Dp[h];
  // Rows in batches of RB: a batch's inputs (x, dt, B and C slices) do not depend on the state,
  // so all of them are loaded before the first row is computed -- one memory round trip per
  // batch instead of one per row; the rows are then run one after another as single steps.
  constexpr int RB = 4;
  for (int t0 = 0; t0 < L; t0 += RB) {
    float xr[RB], dtr[RB], br[RB][NPL], cr[RB][NPL];
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const int t = t0 + r;
      if (t < L) {
        const int64_t row = static_cast<int64_t>(t) * xbc_stride;
        xr[r] = ld<TX>(xbc, row + static_cast<int64_t>(h) * P + p);
        dtr[r] = ld<TD>(dt, static_cast<int64_t>(t) * dt_stride + h);
        const int64_t bo = row + I + static_cast<int64_t>(g) * N + lane * NPL;
        const int64_t co = row + I + static_cast<int64_t>(G) * N + static_cast<int64_t>(g) * N + lane * NPL;
        if constexpr (NPL % 4 == 0) {             // 4 consecutive values per vector load (the host
#pragma unroll                                       // checked 4-element alignment of xbc rows)
          for (int i = 0; i < NPL; i += 4) {
            ld4<TX>(xbc, bo + i, &br[r][i]);
            ld4<TX>(xbc, co + i, &cr[r][i]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < NPL; ++i) {
            br[r][i] = ld<TX>(xbc, bo + i);
            cr[r][i] = ld<TX>(xbc, co + i);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const int t = t0 + r;
      if (t >= L) break;
      const float x = xr[r];
      const float dtt = fminf(fmaxf(softplus_f(dtr[r] + dbias), dt_min), dt_max);
      const float dA = expf(dtt * A);
      const float dx = dtt * x;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        st[i] = fmaf(st[i], dA, dx * br[r][i]);
        acc = fmaf(st[i], cr[r][i], acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0)
        reinterpret_cast<TY*>(y)[static_cast<int64_t>(t) * I + static_cast<int64_t>(h) * P + p] =
            hsd::from_f32<TY>(fmaf(Dh, x, acc));
      if (last_only && t != L - 1) continue;       // prefill: the final state only, in states[0]
      float* dst = states + static_cast<int64_t>(last_only ? 0 : t) * H * P * N + sbase;
      if constexpr (NPL % 4 == 0) {
#pragma unroll
        for (int i = 0; i < NPL; i += 4) *reinterpret_cast<float4*>(dst + i) = make_float4(st[i], st[i + 1], st[i + 2], st[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < NPL; ++i) dst[i] = st[i];
      }
    }
  }
}

// The copying rollback: the kept row's state (float4 pieces) and the conv window (bytes) in one
// grid-stride launch.
__global__ void __launch_bounds__(256) rollback_copy_kernel(const float4* __restrict__ src_state,
                                                            float4* __restrict__ dst_state, int64_t n4,
                                                            const unsigned char* __restrict__ src_win,
                                                            unsigned char* __restrict__ dst_win, int64_t nwin) {
  hsd::pdl_launch_dependents();
  hsd::pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride)
    dst_state[i] = src_state[i];
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nwin; i += stride)
    dst_win[i] = src_win[i];
}

template <typename TI, typename TW>
int conv_dispatch_out(int out_dtype, dim3 grid, cudaStream_t st, const void* conv_in, int64_t in_stride,
                      const void* conv_state, const void* w, const void* bias, void* out, void* padded, int L, int C,
                      const int* n_keep, int rows) {
  switch (out_dtype) {
    case HSD_F32: hsd::launch_pdl(conv_verify_kernel<TI, TW, float>, dim3(grid), dim3(256), 0, st, conv_in, in_stride, conv_state, w, bias, out, padded, L, C, n_keep, rows); break;
    case HSD_F16: hsd::launch_pdl(conv_verify_kernel<TI, TW, __half>, dim3(grid), dim3(256), 0, st, conv_in, in_stride, conv_state, w, bias, out, padded, L, C, n_keep, rows); break;
    case HSD_BF16: hsd::launch_pdl(conv_verify_kernel<TI, TW, __nv_bfloat16>, dim3(grid), dim3(256), 0, st, conv_in, in_stride, conv_state, w, bias, out, padded, L, C, n_keep, rows); break;
    default: return hsd::set_error(HSD_ERR_DTYPE, "hsd_mamba_conv_verify: out_dtype %d", out_dtype);
  }
  return hsd::check_launch("hsd_mamba_conv_verify");
}

template <typename TI>
int conv_dispatch_w(int w_dtype, int out_dtype, dim3 grid, cudaStream_t st, const void* conv_in, int64_t in_stride,
                    const void* conv_state, const void* w, const void* bias, void* out, void* padded, int L, int C,
                    const int* n_keep, int rows) {
  switch (w_dtype) {
    case HSD_F32: return conv_dispatch_out<TI, float>(out_dtype, grid, st, conv_in, in_stride, conv_state, w, bias, out, padded, L, C, n_keep, rows);
    case HSD_BF16: return conv_dispatch_out<TI, __nv_bfloat16>(out_dtype, grid, st, conv_in, in_stride, conv_state, w, bias, out, padded, L, C, n_keep, rows);
  }
  return hsd::set_error(HSD_ERR_DTYPE, "hsd_mamba_conv_verify: w_dtype %d (f32 or bf16)", w_dtype);
}

template <typename TX, typename TD, typename TY>
int ssm_dispatch_n(int N, dim3 grid, cudaStream_t st, const void* xbc, int64_t xbc_stride, const void* dt,
                   int64_t dt_stride, const float* A_log, const float* Dp, const float* dt_bias, float dt_min,
                   float dt_max, const float* state0, float* states, void* y, int L, int H, int P, int G,
                   int last_only, const int* n_keep, int rows) {
  switch (N) {
    case 32: hsd::launch_pdl(ssm_verify_kernel<TX, TD, TY, 1>, dim3(grid), dim3(256), 0, st, xbc, xbc_stride, dt, dt_stride, A_log, Dp, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, N, last_only, n_keep, rows); break;
    case 64: hsd::launch_pdl(ssm_verify_kernel<TX, TD, TY, 2>, dim3(grid), dim3(256), 0, st, xbc, xbc_stride, dt, dt_stride, A_log, Dp, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, N, last_only, n_keep, rows); break;
    case 128: hsd::launch_pdl(ssm_verify_kernel<TX, TD, TY, 4>, dim3(grid), dim3(256), 0, st, xbc, xbc_stride, dt, dt_stride, A_log, Dp, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, N, last_only, n_keep, rows); break;
    case 256: hsd::launch_pdl(ssm_verify_kernel<TX, TD, TY, 8>, dim3(grid), dim3(256), 0, st, xbc, xbc_stride, dt, dt_stride, A_log, Dp, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, N, last_only, n_keep, rows); break;
    default: return hsd::set_error(HSD_ERR_SHAPE, "hsd_mamba_ssm_verify: N must be 32, 64, 128 or 256 (got %d)", N);
  }
  return hsd::check_launch("hsd_mamba_ssm_verify");
}

template <typename TX>
int ssm_dispatch(int dt_dtype, int y_dtype, int N, dim3 grid, cudaStream_t st, const void* xbc, int64_t xbc_stride,
                 const void* dt, int64_t dt_stride, const float* A_log, const float* Dp, const float* dt_bias,
                 float dt_min, float dt_max, const float* state0, float* states, void* y, int L, int H, int P,
                 int G, int last_only, const int* n_keep, int rows) {
#define HSD_SSM_Y(TD)                                                                                            \
  switch (y_dtype) {                                                                                           \
    case HSD_F32: return ssm_dispatch_n<TX, TD, float>(N, grid, st, xbc, xbc_stride, dt, dt_stride, A_log, Dp, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, last_only, n_keep, rows); \
    case HSD_BF16: return ssm_dispatch_n<TX, TD, __nv_bfloat16>(N, grid, st, xbc, xbc_stride, dt, dt_stride, A_log, Dp, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, last_only, n_keep, rows); \
  }                                                                                                            \
  return hsd::set_error(HSD_ERR_DTYPE, "hsd_mamba_ssm_verify: y_dtype %d (f32 or bf16)", y_dtype);
  switch (dt_dtype) {
    case HSD_F32: { HSD_SSM_Y(float) }
    case HSD_BF16: { HSD_SSM_Y(__nv_bfloat16) }
  }
#undef HSD_SSM_Y
  return hsd::set_error(HSD_ERR_DTYPE, "hsd_mamba_ssm_verify: dt_dtype %d (f32 or bf16)", dt_dtype);
}

}  // namespace

namespace {

int conv_impl(const char* who, const void* conv_in, int in_dtype, int64_t in_stride, const void* conv_state,
              const void* w, int w_dtype, const void* bias, void* out, int out_dtype, void* padded, int L, int C,
              int K, const int* n_keep, int rows, void* stream) {
  if (!conv_in || !w || !out || !padded) return hsd::set_error(HSD_ERR_ARG, "%s: null pointer", who);
  if (L < 1 || C < 1 || K != 4 || in_stride < C)
    return hsd::set_error(HSD_ERR_SHAPE, "%s: need L >= 1, K == 4, in_stride >= C", who);
  dim3 grid((C + 255) / 256);
  cudaStream_t st = hsd::as_stream(stream);
  switch (in_dtype) {
    case HSD_F32: return conv_dispatch_w<float>(w_dtype, out_dtype, grid, st, conv_in, in_stride, conv_state, w, bias, out, padded, L, C, n_keep, rows);
    case HSD_BF16: return conv_dispatch_w<__nv_bfloat16>(w_dtype, out_dtype, grid, st, conv_in, in_stride, conv_state, w, bias, out, padded, L, C, n_keep, rows);
  }
  return hsd::set_error(HSD_ERR_DTYPE, "%s: in_dtype %d (f32 or bf16)", who, in_dtype);
}

int ssm_impl(const char* who, const void* xbc, int x_dtype, int64_t xbc_stride, const void* dt, int dt_dtype,
             int64_t dt_stride, const float* A_log, const float* D, const float* dt_bias, float dt_min, float dt_max,
             const float* state0, float* states, void* y, int y_dtype, int L, int H, int P, int G, int N,
             int last_only, const int* n_keep, int rows, void* stream) {
  if (!xbc || !dt || !A_log || !D || !dt_bias || !states || !y)
    return hsd::set_error(HSD_ERR_ARG, "%s: null pointer", who);
  if (L < 1 || H < 1 || P < 1 || G < 1 || H % G != 0 || xbc_stride < static_cast<int64_t>(H) * P + 2 * G * N)
    return hsd::set_error(HSD_ERR_SHAPE, "%s: bad shape (H %% G == 0, xbc_stride >= H*P + 2*G*N)", who);
  if (!hsd::aligned(states, 16) || (state0 && !hsd::aligned(state0, 16)))
    return hsd::set_error(HSD_ERR_ALIGN, "%s: states must be 16-byte aligned", who);
  const int xb = x_dtype == HSD_F32 ? 4 : 2;
  if (N >= 128 && (!hsd::aligned(xbc, 4 * xb) || (xbc_stride * xb) % (4 * xb) != 0 || (static_cast<int64_t>(H) * P) % 4 != 0))
    return hsd::set_error(HSD_ERR_ALIGN, "%s: xbc rows must start on 4-element boundaries (N >= 128 uses vector loads)", who);
  const int64_t warps = static_cast<int64_t>(H) * P;
  dim3 grid(static_cast<unsigned>((warps * 32 + 255) / 256));
  cudaStream_t st = hsd::as_stream(stream);
  switch (x_dtype) {
    case HSD_F32: return ssm_dispatch<float>(dt_dtype, y_dtype, N, grid, st, xbc, xbc_stride, dt, dt_stride, A_log, D, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, last_only, n_keep, rows);
    case HSD_BF16: return ssm_dispatch<__nv_bfloat16>(dt_dtype, y_dtype, N, grid, st, xbc, xbc_stride, dt, dt_stride, A_log, D, dt_bias, dt_min, dt_max, state0, states, y, L, H, P, G, last_only, n_keep, rows);
  }
  return hsd::set_error(HSD_ERR_DTYPE, "%s: x_dtype %d (f32 or bf16)", who, x_dtype);
}

}  // namespace

extern "C" int hsd_mamba_conv_verify(const void* conv_in, int in_dtype, int64_t in_stride, const void* conv_state,
                                     const void* w, int w_dtype, const void* bias, void* out, int out_dtype,
                                     void* padded, int L, int C, int K, void* stream) {
  return conv_impl("hsd_mamba_conv_verify", conv_in, in_dtype, in_stride, conv_state, w, w_dtype, bias, out,
                   out_dtype, padded, L, C, K, nullptr, 0, stream);
}

extern "C" int hsd_mamba_ssm_verify(const void* xbc, int x_dtype, int64_t xbc_stride, const void* dt, int dt_dtype,
                                    int64_t dt_stride, const float* A_log, const float* D, const float* dt_bias,
                                    float dt_min, float dt_max, const float* state0, float* states, void* y,
                                    int y_dtype, int L, int H, int P, int G, int N, int last_only, void* stream) {
  return ssm_impl("hsd_mamba_ssm_verify", xbc, x_dtype, xbc_stride, dt, dt_dtype, dt_stride, A_log, D, dt_bias,
                  dt_min, dt_max, state0, states, y, y_dtype, L, H, P, G, N, last_only, nullptr, 0, stream);
}

extern "C" int hsd_mamba_conv_step(const void* conv_in, int in_dtype, int64_t in_stride, void* padded,
                                   const int* n_keep, int rows, const void* w, int w_dtype, const void* bias,
                                   void* out, int out_dtype, int L, int C, int K, void* stream) {
  if (!n_keep || rows < 1 || L > rows)
    return hsd::set_error(HSD_ERR_ARG, "hsd_mamba_conv_step: need n_keep and 1 <= L <= rows (L=%d rows=%d)", L, rows);
  return conv_impl("hsd_mamba_conv_step", conv_in, in_dtype, in_stride, nullptr, w, w_dtype, bias, out, out_dtype,
                   padded, L, C, K, n_keep, rows, stream);
}

extern "C" int hsd_mamba_ssm_step(const void* xbc, int x_dtype, int64_t xbc_stride, const void* dt, int dt_dtype,
                                  int64_t dt_stride, const float* A_log, const float* D, const float* dt_bias,
                                  float dt_min, float dt_max, float* states, const int* n_keep, int rows, void* y,
                                  int y_dtype, int L, int H, int P, int G, int N, void* stream) {
  if (!n_keep || rows < 1 || L > rows)
    return hsd::set_error(HSD_ERR_ARG, "hsd_mamba_ssm_step: need n_keep and 1 <= L <= rows (L=%d rows=%d)", L, rows);
  return ssm_impl("hsd_mamba_ssm_step", xbc, x_dtype, xbc_stride, dt, dt_dtype, dt_stride, A_log, D, dt_bias, dt_min,
                  dt_max, nullptr, states, y, y_dtype, L, H, P, G, N, 0, n_keep, rows, stream);
}

extern "C" int hsd_mamba_rollback(const float* states, const void* padded, int elem_bytes, int n_keep, int L, int H,
                                  int P, int N, int C, int K, float* state_out, void* conv_out, void* stream) {
  if (!states || !padded || !state_out || !conv_out) return hsd::set_error(HSD_ERR_ARG, "hsd_mamba_rollback: null pointer");
  if (n_keep < 1 || n_keep > L || elem_bytes < 1 || K < 1)
    return hsd::set_error(HSD_ERR_ARG, "hsd_mamba_rollback: need 1 <= n_keep <= L (got n_keep=%d L=%d)", n_keep, L);
  cudaStream_t st = hsd::as_stream(stream);
  const int64_t snum = static_cast<int64_t>(H) * P * N;
  if (snum % 4 != 0 || !hsd::aligned(states, 16) || !hsd::aligned(state_out, 16))
    return hsd::set_error(HSD_ERR_ALIGN, "hsd_mamba_rollback: states / state_out must be 16-byte aligned, H*P*N %% 4 == 0");
  const int64_t nwin = static_cast<int64_t>(K - 1) * C * elem_bytes;
  const int64_t n4 = snum / 4;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n4 + 255) / 256, 148 * 8));
  cudaError_t e = hsd::launch_pdl(rollback_copy_kernel, dim3(grid), dim3(256), 0, st,
                                  reinterpret_cast<const float4*>(states + static_cast<int64_t>(n_keep - 1) * snum),
                                  reinterpret_cast<float4*>(state_out), n4,
                                  static_cast<const unsigned char*>(padded) + static_cast<int64_t>(n_keep) * C * elem_bytes,
                                  static_cast<unsigned char*>(conv_out), nwin);
  return hsd::check_cuda(e, "hsd_mamba_rollback");
}
