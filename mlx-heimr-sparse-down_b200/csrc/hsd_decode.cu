// Sparse MoE down projection for decode on the neuron-major layout (hsd/decode.py).
//
//   y[b, o] = sum_k gains[b,k] * sum_{i : h[b,k,i] != 0} h[b,k,i] * W_{sel[b,k]}[o, i]
//           + gains[b,topk]   * sum_{i : hs[b,i] != 0}  hs[b,i]  * Ws[o, i]
//   W[o, i] = s[i/64, o] * q[i, o] + b[i/64, o]           (affine 4-bit, group 64)
//
// Work split (one token = one row b of h):
//   The token's 64-neuron groups are listed slot by slot (topk routed experts, then the
//   shared expert): GT = topk*F/64 + FS/64 groups (232 at the reference shapes). The D
//   outputs are cut into chunks of C outputs (C/2 contiguous bytes of every neuron row).
//   A thread-block CLUSTER of 8 CTAs owns one (token, chunk); CTA `rank` of the cluster
//   owns groups [rank*GT/8, (rank+1)*GT/8) -- at the reference shapes exactly one routed
//   expert or one half of the shared expert (29 groups) each. The 8 partial outputs are
//   summed through distributed shared memory in a fixed rank order, so the result is
//   deterministic and no scratch memory, atomics or second kernel is needed.
//
// Per CTA and batch of up to 32 groups:
//   1. each warp reads the h of its groups (64 values each) and builds the group's live
//      mask with two warp ballots; warp 0 scans the live counts;
//   2. the live rows are compacted (ballot prefix popcounts) into an ascending list;
//   3. 16-byte cp.async copies stage, for live groups only, the chunk of the group's
//      scales and biases, and for live rows only, the row's C/2-byte chunk -- all copies
//      of a batch are in flight at once;
//   4. thread (word wp, row lane rl) walks rows rl, rl+NRL, ... accumulating, per 64-group,
//      acc'[n] = sum h * (1 + q_n/16) and hsum = sum h in fp32, and folds each finished group
//      in as out[n] += g * (16*s[n]*(acc'[n] - hsum) + b[n]*hsum) -- the same affine algebra as
//      the reference (s * sum(h q) + b * sum(h)); 1 + q/16 is built exactly from the nibble
//      by bit operations, which spares an integer-to-float conversion per weight.
//   5. the NRL row lanes are reduced in shared memory in a fixed order.
#include <cooperative_groups.h>

#include "hsd_common.cuh"

namespace cg = cooperative_groups;

HSD_DEFINE_STATUS(decode)

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCluster = 8;    // CTAs per (token, chunk)
constexpr int kGB = 32;        // groups per batch
constexpr int kRB = 512;       // staged rows per sub-batch
constexpr int kGS = 64;        // quantisation group size

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
  int NR;    // columns of h: topk*F + FS
  int GT;    // groups per token
  int NW;    // words per neuron row: D/8
};

template <int C>
struct DecodeSmem {
  static constexpr int NWC = C / 8;             // words of one row in a chunk
  float hs[kGB * kGS];                          // the batch's h values (fp32)
  uint32_t stage[kRB * NWC];                    // staged row chunks
  uint16_t meta_s[kGB * C];                     // staged scale chunks (16-bit)
  uint16_t meta_b[kGB * C];                     // staged bias chunks
  uint16_t rows[kGB * kGS];                     // compacted live rows: (group in batch) << 6 | neuron
  unsigned long long gmask[kGB];
  int gcnt[kGB], goff[kGB + 1];
  int gsrc[kGB];                                // expert id, -1 = shared expert, -2 = invalid
  int gloc[kGB];                                // the group's index inside its expert
  float ggain[kGB];
  float part[C];                                // this CTA's partial output chunk
};

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

template <typename HT>
__device__ __forceinline__ float load_h(const void* h, int64_t idx) {
  return hsd::to_f32<HT>(reinterpret_cast<const HT*>(h)[idx]);
}

template <typename HT, typename ST, typename YT, int C>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads)
    sparse_down_decode_kernel(const DecodeParams p) {
  constexpr int NWC = C / 8;
  constexpr int NRL = kThreads / NWC;            // row lanes
  extern __shared__ __align__(16) unsigned char smem_raw[];
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

  const int wp = tid % NWC;                       // word of the chunk this thread owns
  const int rl = tid / NWC;                       // row lane
  const bool active = wp < nwc;

  float out[8];
#pragma unroll
  for (int n = 0; n < 8; ++n) out[n] = 0.f;

  for (int gb0 = g_lo; gb0 < g_hi; gb0 += kGB) {
    const int ng = min(kGB, g_hi - gb0);
    // ---- 1. h, live masks and counts, one warp per group
    for (int gi = warp; gi < ng; gi += kWarps) {
      const int G = gb0 + gi;
      int slot, gl, src;
      if (G < p.topk * GF) {
        slot = G / GF;
        gl = G - slot * GF;
        src = (lane == 0) ? __ldg(p.sel + static_cast<int64_t>(b) * p.topk + slot) : 0;
        src = __shfl_sync(0xffffffffu, src, 0);
        if (src < 0 || src >= p.E) {
          if (lane == 0) hsd_flag_decode(HSD_ERR_INDEX);
          src = -2;
        }
      } else {
        slot = p.topk;
        gl = G - p.topk * GF;
        src = -1;
      }
      const int64_t hcol = static_cast<int64_t>(b) * p.NR + static_cast<int64_t>(slot) * p.F +
                           static_cast<int64_t>(gl) * kGS;
      float v0 = 0.f, v1 = 0.f;
      if (src != -2) {
        v0 = load_h<HT>(p.h, hcol + lane);
        v1 = load_h<HT>(p.h, hcol + 32 + lane);
      }
      S.hs[gi * kGS + lane] = v0;
      S.hs[gi * kGS + 32 + lane] = v1;
      const unsigned long long m = ballot64(v0 != 0.f, v1 != 0.f);
      if (lane == 0) {
        S.gmask[gi] = m;
        S.gcnt[gi] = __popcll(m);
        S.gsrc[gi] = src;
        S.gloc[gi] = gl;
        S.ggain[gi] = __ldg(p.gains + static_cast<int64_t>(b) * (p.topk + 1) + slot);
      }
    }
    __syncthreads();
    // ---- 2. scan the counts (warp 0), then compact the live rows (one warp per group)
    if (warp == 0) {
      const int c = (lane < ng) ? S.gcnt[lane] : 0;
      int x = c;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
      }
      if (lane < ng) S.goff[lane] = x - c;
      if (lane == 31) S.goff[ng] = x;   // (lanes >= ng add zero, so lane 31 holds the total)
    }
    __syncthreads();
    const int nrows = S.goff[ng];
    for (int gi = warp; gi < ng; gi += kWarps) {
      const unsigned long long m = S.gmask[gi];
      const int base = S.goff[gi];
      if ((m >> lane) & 1ull) S.rows[base + live_prefix(m, lane)] = static_cast<uint16_t>((gi << 6) | lane);
      if ((m >> (lane + 32)) & 1ull)
        S.rows[base + live_prefix(m, lane + 32)] = static_cast<uint16_t>((gi << 6) | (lane + 32));
    }
    __syncthreads();

    // ---- 3./4. stage and accumulate, sub-batches of kRB rows
    int gcur = -1;
    float acc[8], hsum = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) acc[n] = 0.f;

    auto flush = [&](int gi) {
      const float g = S.ggain[gi];
      if (p.loadsc) {
        const uint4 s4 = *reinterpret_cast<const uint4*>(&S.meta_s[gi * C + wp * 8]);
        const uint4 b4 = *reinterpret_cast<const uint4*>(&S.meta_b[gi * C + wp * 8]);
        const uint32_t sw[4] = {s4.x, s4.y, s4.z, s4.w};
        const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const float s = hsd::bits16_to_f32<ST>(static_cast<uint16_t>(sw[n >> 1] >> (16 * (n & 1))));
          const float bb = hsd::bits16_to_f32<ST>(static_cast<uint16_t>(bw[n >> 1] >> (16 * (n & 1))));
          out[n] = fmaf(g, fmaf(16.f * s, acc[n] - hsum, bb * hsum), out[n]);
        }
      } else {
#pragma unroll
        for (int n = 0; n < 8; ++n) out[n] = fmaf(g, fmaf(16.f, acc[n] - hsum, hsum), out[n]);
      }
    };

    for (int r0 = 0; r0 < nrows; r0 += kRB) {
      const int rn = min(kRB, nrows - r0);
      if (r0 == 0 && p.loadsc) {                 // the batch's live groups' scale / bias chunks
        // one 16-byte piece = the 8 scales (or biases) of one word's 8 outputs
        for (int t = tid; t < ng * 2 * nwc; t += kThreads) {
          const int gi = t / (2 * nwc);
          const int rem = t - gi * 2 * nwc;
          const int which = rem / nwc, pc = rem - which * nwc;
          if (S.gcnt[gi] == 0) continue;
          const int src = S.gsrc[gi];
          const int64_t grow = (src >= 0) ? static_cast<int64_t>(src) * GF + S.gloc[gi] : S.gloc[gi];
          const uint16_t* base = (src >= 0) ? (which ? p.pb : p.ps) : (which ? p.spb : p.sps);
          const uint16_t* g = base + grow * p.D + static_cast<int64_t>(w0 + pc) * 8;
          uint16_t* d = (which ? S.meta_b : S.meta_s) + gi * C + pc * 8;
          hsd::cp_async16(d, g);
        }
      }
      {                                          // the sub-batch's live row chunks
        const int pieces = nwc / 4;              // 16-byte pieces per row chunk
        for (int t = tid; t < rn * pieces; t += kThreads) {
          const int r = t / pieces, pc = t - r * pieces;
          const int code = S.rows[r0 + r];
          const int gi = code >> 6, j = code & 63;
          const int src = S.gsrc[gi];
          const int64_t neuron = static_cast<int64_t>(S.gloc[gi]) * kGS + j;
          const uint32_t* g = (src >= 0) ? p.pw + (static_cast<int64_t>(src) * p.F + neuron) * p.NW
                                         : p.spw + neuron * p.NW;
          hsd::cp_async16(&S.stage[r * NWC + pc * 4], g + w0 + pc * 4);
        }
      }
      hsd::cp_async_commit();
      hsd::cp_async_wait_all();
      __syncthreads();
      if (active) {
        for (int r = rl; r < rn; r += NRL) {
          const int code = S.rows[r0 + r];
          const int gi = code >> 6;
          const float hv = S.hs[gi * kGS + (code & 63)];
          const uint32_t q = S.stage[r * NWC + wp];
          if (gi != gcur) {
            if (gcur >= 0) flush(gcur);
            gcur = gi;
            hsum = 0.f;
#pragma unroll
            for (int n = 0; n < 8; ++n) acc[n] = 0.f;
          }
          hsum += hv;
          acc[0] = fmaf(hv, nib_unit<0>(q), acc[0]);
          acc[1] = fmaf(hv, nib_unit<1>(q), acc[1]);
          acc[2] = fmaf(hv, nib_unit<2>(q), acc[2]);
          acc[3] = fmaf(hv, nib_unit<3>(q), acc[3]);
          acc[4] = fmaf(hv, nib_unit<4>(q), acc[4]);
          acc[5] = fmaf(hv, nib_unit<5>(q), acc[5]);
          acc[6] = fmaf(hv, nib_unit<6>(q), acc[6]);
          acc[7] = fmaf(hv, nib_unit<7>(q), acc[7]);
        }
      }
      __syncthreads();                           // stage is rewritten by the next sub-batch
    }
    if (active && gcur >= 0) flush(gcur);
    __syncthreads();                             // meta / hs / rows are rewritten by the next batch
  }

  // ---- 5. reduce the row lanes (fixed order) into S.part, reusing the stage buffer
  float* red = reinterpret_cast<float*>(S.stage);   // [NRL][C] fp32 (NRL*C = 2*kThreads*... fits)
#pragma unroll
  for (int n = 0; n < 8; ++n) red[rl * C + wp * 8 + n] = out[n];
  __syncthreads();
  for (int o = tid; o < C; o += kThreads) {
    float t = 0.f;
    for (int l = 0; l < NRL; ++l) t += red[l * C + o];
    S.part[o] = t;
  }
  // ---- 6. the cluster's 8 partials, summed in rank order through DSMEM
  cluster.sync();
  constexpr int per = C / kCluster;
  for (int i = tid; i < per; i += kThreads) {
    const int o = rank * per + i;
    if (o < nwc * 8) {
      float t = 0.f;
#pragma unroll
      for (int q = 0; q < kCluster; ++q) t += cluster.map_shared_rank(S.part, q)[o];
      const int64_t yi = static_cast<int64_t>(b) * p.D + static_cast<int64_t>(w0) * 8 + o;
      if (p.resid) t += hsd::to_f32<YT>(reinterpret_cast<const YT*>(p.resid)[yi]);
      reinterpret_cast<YT*>(p.y)[yi] = hsd::from_f32<YT>(t);
    }
  }
  cluster.sync();                                // keep this CTA's smem alive for the readers
}

// ---- active-index sets, the same ballot compaction per (token, slot)
template <typename HT>
__global__ void __launch_bounds__(kThreads) live_rows_kernel(const void* h, int32_t* live,
                                                             int32_t* count, int F, int FS, int topk) {
  const int slot = blockIdx.x, b = blockIdx.y;
  const int width = (slot < topk) ? F : FS;
  const int NR = topk * F + FS;
  const int maxw = max(F, FS);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ int wcnt[kThreads / 32];
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

template <typename HT, typename ST, typename YT, int C>
int launch_decode(const DecodeParams& p, cudaStream_t st) {
  auto kern = sparse_down_decode_kernel<HT, ST, YT, C>;
  const size_t smem = sizeof(DecodeSmem<C>);
  static_assert(sizeof(float) * (kThreads / (C / 8)) * C <= sizeof(uint32_t) * kRB * (C / 8),
                "row-lane reduction must fit in the stage buffer");
  static int configured_device = -1;           // the attribute is set once per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_device != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return hsd::check_cuda(e, "hsd_sparse_down_decode: smem attribute");
    configured_device = dev;
  }
  const int nch = (p.NW + (C / 8) - 1) / (C / 8);
  dim3 grid(nch * kCluster, p.B);
  kern<<<grid, kThreads, smem, st>>>(p);
  return hsd::check_launch("hsd_sparse_down_decode");
}

template <typename HT, typename ST>
int dispatch_y(int y_dtype, const DecodeParams& p, cudaStream_t st) {
  switch (y_dtype) {
    case HSD_F32: return launch_decode<HT, ST, float, 128>(p, st);
    case HSD_F16: return launch_decode<HT, ST, __half, 128>(p, st);
    case HSD_BF16: return launch_decode<HT, ST, __nv_bfloat16, 128>(p, st);
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

extern "C" int hsd_sparse_down_decode(const void* h, int h_dtype, const int32_t* sel,
                                      const float* gains, const uint32_t* pw, const void* ps,
                                      const void* pb, int s_dtype, const uint32_t* spw,
                                      const void* sps, const void* spb, const void* resid, void* y,
                                      int y_dtype, int B, int D, int F, int FS, int topk, int E,
                                      int loadsc, void* stream) {
  if (!h || !sel || !gains || !pw || !ps || !pb || !spw || !sps || !spb || !y)
    return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_decode: null pointer");
  if (B < 1 || B > 65535 || D < 32 || D % 32 != 0 || F < 64 || F % 64 != 0 || FS < 64 ||
      FS % 64 != 0 || topk < 1 || E < 1)
    return hsd::set_error(HSD_ERR_SHAPE,
                          "hsd_sparse_down_decode: need 1<=B<=65535, D%%32==0, F%%64==0, FS%%64==0, "
                          "topk>=1, E>=1 (got B=%d D=%d F=%d FS=%d topk=%d E=%d)",
                          B, D, F, FS, topk, E);
  const long long NR = static_cast<long long>(topk) * F + FS;
  if (NR > (1ll << 30) || static_cast<long long>(E) * F * (D / 8) > (1ll << 40))
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_sparse_down_decode: sizes too large");
  const void* ptr16[] = {pw, ps, pb, spw, sps, spb};
  for (const void* q : ptr16)
    if (!hsd::aligned(q, 16))
      return hsd::set_error(HSD_ERR_ALIGN, "hsd_sparse_down_decode: weight pointers must be 16-byte aligned");
  DecodeParams p;
  p.h = h; p.sel = sel; p.gains = gains; p.pw = pw;
  p.ps = static_cast<const uint16_t*>(ps); p.pb = static_cast<const uint16_t*>(pb);
  p.spw = spw; p.sps = static_cast<const uint16_t*>(sps); p.spb = static_cast<const uint16_t*>(spb);
  p.resid = resid; p.y = y;
  p.B = B; p.D = D; p.F = F; p.FS = FS; p.topk = topk; p.E = E; p.loadsc = loadsc ? 1 : 0;
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

extern "C" int hsd_decode_live_rows(const void* h, int h_dtype, int32_t* live, int32_t* count, int B,
                                    int F, int FS, int topk, void* stream) {
  if (!h || !live || !count) return hsd::set_error(HSD_ERR_ARG, "hsd_decode_live_rows: null pointer");
  if (B < 1 || B > 65535 || F < 64 || F % 64 != 0 || FS < 64 || FS % 64 != 0 || topk < 1)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_decode_live_rows: bad shape");
  dim3 grid(topk + 1, B);
  cudaStream_t st = hsd::as_stream(stream);
  switch (h_dtype) {
    case HSD_F32: live_rows_kernel<float><<<grid, kThreads, 0, st>>>(h, live, count, F, FS, topk); break;
    case HSD_F16: live_rows_kernel<__half><<<grid, kThreads, 0, st>>>(h, live, count, F, FS, topk); break;
    case HSD_BF16:
      live_rows_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(h, live, count, F, FS, topk);
      break;
    default: return hsd::set_error(HSD_ERR_DTYPE, "hsd_decode_live_rows: h_dtype %d", h_dtype);
  }
  return hsd::check_launch("hsd_decode_live_rows");
}
