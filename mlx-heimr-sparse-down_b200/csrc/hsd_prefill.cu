// Prefill kernels (hsd/prefill.py): the expert-sorted tile order, the per-tile live unions,
// the A-operand gather, the partial-sum reduce. The tensor-core GEMM is in hsd_prefill_gemm.cu.
//
// Tile order (hsd/prefill.py:247-278): the (token, expert-slot) pairs of a chunk, slot id
// t*topk + k, sorted by expert and cut into tiles of tt slots of one expert, then the shared
// expert's tiles of tt tokens. The tile count is FIXED by (T, topk, E, tt) -- never by the
// routing -- so nothing is read back to the host: routed tiles the routing does not fill
// carry expert -1, padding slots are -1. Inside an expert the slots keep ascending slot
// order (a stable sort).
#include <algorithm>

#include "hsd_common.cuh"
#include "hsd_prefill.cuh"

HSD_DEFINE_STATUS(prefill)

namespace {

constexpr int kTileThreads = 1024;
constexpr int kTileWarps = kTileThreads / 32;
constexpr int kMaxExperts = 256;

// One CTA: histogram of the experts, tile bases, then stable per-expert ranks chunk by chunk
// of 1024 slots: a slot's rank = its expert's count in earlier chunks + in earlier warps of
// this chunk (a [warp][expert] table, scanned over warps) + its peers below it in its warp
// (warp match). Then the slot scatter and the tile experts.
__global__ void __launch_bounds__(kTileThreads) build_tiles_kernel(const int32_t* __restrict__ sel,
                                                                   int T, int topk, int E, int tt,
                                                                   int nt_routed, int nt_shared, int T_shared,
                                                                   const int* __restrict__ nslots_dev,
                                                                   int32_t* __restrict__ tile_e,
                                                                   int32_t* __restrict__ tile_slot) {
  __shared__ int cnt[kMaxExperts];
  __shared__ int tbase[kMaxExperts];
  __shared__ int running[kMaxExperts];
  __shared__ int before[kMaxExperts];           // running[] at the start of the chunk
  __shared__ uint16_t tab[kTileWarps][kMaxExperts];   // per chunk: slots of expert e in warp w
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nslots = nslots_dev ? min(max(*nslots_dev, 0), T * topk) : T * topk;
  const int NT = nt_routed + nt_shared;
  for (int i = tid; i < E; i += kTileThreads) {
    cnt[i] = 0;
    running[i] = 0;
  }
  for (int i = tid; i < NT; i += kTileThreads) tile_e[i] = -1;
  for (int i = tid; i < NT * tt; i += kTileThreads) tile_slot[i] = -1;
  __syncthreads();
  for (int j = tid; j < nslots; j += kTileThreads) {
    const int e = sel[j];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
    else hsd_flag_prefill(HSD_ERR_INDEX);      // the slot is dropped: its token's y is unspecified
  }
  __syncthreads();
  if (tid == 0) {                                 // E <= 256: a serial scan is short
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      tbase[e] = acc;
      acc += (cnt[e] + tt - 1) / tt;
    }
  }
  __syncthreads();
  for (int e = tid; e < E; e += kTileThreads) {
    const int n = (cnt[e] + tt - 1) / tt;
    for (int i = 0; i < n && tbase[e] + i < nt_routed; ++i) tile_e[tbase[e] + i] = e;
  }
  for (int c0 = 0; c0 < nslots; c0 += kTileThreads) {
    for (int i = tid; i < kTileWarps * E; i += kTileThreads) tab[i / E][i % E] = 0;
    __syncthreads();
    const int j = c0 + tid;
    const int e = (j < nslots) ? sel[j] : -1;
    const bool ok = e >= 0 && e < E;
    const unsigned peers = __match_any_sync(0xffffffffu, ok ? e : -1);
    const int below = __popc(peers & ((1u << lane) - 1u));
    if (ok && below == 0) tab[warp][e] = static_cast<uint16_t>(__popc(peers));
    __syncthreads();
    for (int ex = tid; ex < E; ex += kTileThreads) {   // exclusive scan over warps
      int acc = 0;
      for (int w = 0; w < kTileWarps; ++w) {
        const int v = tab[w][ex];
        tab[w][ex] = static_cast<uint16_t>(acc);
        acc += v;
      }
      before[ex] = running[ex];
      running[ex] += acc;
    }
    __syncthreads();
    if (ok) {
      const int rank = before[e] + tab[warp][e] + below;
      const int t = tbase[e] + rank / tt;
      if (t < nt_routed) tile_slot[t * tt + rank % tt] = j;
    }
    __syncthreads();
  }
  // the shared expert's tiles: tokens 0 .. T_shared-1 in order
  for (int i = tid; i < nt_shared; i += kTileThreads) tile_e[nt_routed + i] = E;
  for (int i = tid; i < nt_shared * tt; i += kTileThreads)
    tile_slot[nt_routed * tt + i] = (i < T_shared) ? i : -1;
}

// Union of live columns per tile (hsd/prefill.py:48-93): one CTA per tile; thread-per-column
// OR over the tile's slots, compacted with a block-wide scan in ascending column order.
template <typename HT>
__global__ void __launch_bounds__(256) build_union_kernel(const HT* __restrict__ h,
                                                          const int32_t* __restrict__ tile_e,
                                                          const int32_t* __restrict__ tile_slot, int tt,
                                                          int F, int FS, int topk, int E, int umax,
                                                          int32_t* __restrict__ ulist,
                                                          int32_t* __restrict__ ucount) {
  const int tile = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ int64_t hoff[1024];
  __shared__ int wsum[8];
  __shared__ int base_s;
  int32_t* out = ulist + static_cast<int64_t>(tile) * umax;
  const int e = tile_e[tile];
  if (e < 0) {
    for (int i = tid; i < umax; i += 256) out[i] = -1;
    if (tid == 0) ucount[tile] = 0;
    return;
  }
  const bool shared = e >= E;
  const int FF = shared ? FS : F;
  const int64_t NR = static_cast<int64_t>(topk) * F + FS;
  for (int m = tid; m < tt; m += 256) {
    const int s = tile_slot[static_cast<int64_t>(tile) * tt + m];
    hoff[m] = (s < 0) ? -1
                      : (shared ? s * NR + static_cast<int64_t>(topk) * F
                                : (s / topk) * NR + static_cast<int64_t>(s % topk) * F);
  }
  if (tid == 0) base_s = 0;
  __syncthreads();
  for (int c0 = 0; c0 < umax; c0 += 256) {
    const int c = c0 + tid;
    bool live = false;
    if (c < FF)
      for (int m = 0; m < tt && !live; ++m) {
        const int64_t o = hoff[m];
        live = o >= 0 && hsd::to_f32<HT>(h[o + c]) != 0.f;
      }
    const unsigned bal = __ballot_sync(0xffffffffu, live);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    int before = base_s;
    for (int w = 0; w < warp; ++w) before += wsum[w];
    if (live) out[before + __popc(bal & ((1u << lane) - 1u))] = c;
    __syncthreads();
    if (tid == 0) {
      int t = 0;
      for (int w = 0; w < 8; ++w) t += wsum[w];
      base_s += t;
    }
    __syncthreads();
  }
  for (int i = base_s + tid; i < umax; i += 256) out[i] = -1;
  if (tid == 0) ucount[tile] = base_s;
}

// A operand: hc[tile*tt + m, c] = fp16(h[slot's columns][c]), c < the tile's K, zero rows for
// padding slots; 8 columns (one 16-byte store) per thread. Rows of empty tiles are skipped.
// Routed slot t*topk + k reads h[t * h_stride + k*F + c]; the shared expert's row of token t
// reads hs[t * hs_stride + c].
// One CTA per (64-column group, tile): its 128 A rows' 64 columns as fp16 (8 lanes a row, 16
// bytes a lane, coalesced both ways), and one byte of the tile's live-K-tile mask,
// kmask[tile][group] = 1 iff any of them is nonzero (rows of mask_row_bytes(kmax) bytes) --
// the tensor-core GEMM skips the K-tiles whose byte is 0 (only zeros to multiply). Every byte a
// non-empty tile's GEMM uses is written here, so the mask needs no clearing.
template <typename HT>
__global__ void __launch_bounds__(256) gather_kernel(const HT* __restrict__ h, int64_t h_stride,
                                                     const int32_t* __restrict__ tile_e,
                                                     const int32_t* __restrict__ tile_slot, int tt,
                                                     int F, int FS, int topk, int E, int kmax,
                                                     __half* __restrict__ hc, uint8_t* __restrict__ kmask,
                                                     const HT* __restrict__ hs, int64_t hs_stride) {
  const int grp = blockIdx.x, tile = blockIdx.y;
  const int e = tile_e[tile];
  if (e < 0) return;
  const bool shared = e >= E;
  const int FF = shared ? FS : F;
  const int c8 = grp * 64 + (threadIdx.x & 7) * 8;
  bool nz = false;
  if (grp * 64 < FF) {
    for (int r = threadIdx.x >> 3; r < tt; r += 32) {
      const int64_t row = static_cast<int64_t>(tile) * tt + r;
      const int s = tile_slot[row];
      __align__(16) __half v[8];
      if (s < 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __float2half_rn(0.f);
      } else {
        const HT* src = shared ? hs + s * hs_stride + c8
                               : h + (s / topk) * h_stride + static_cast<int64_t>(s % topk) * F + c8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[i] = __float2half_rn(hsd::to_f32<HT>(src[i]));
          nz |= (__half_as_ushort(v[i]) & 0x7FFFu) != 0u;
        }
      }
      *reinterpret_cast<uint4*>(hc + row * kmax + c8) = *reinterpret_cast<const uint4*>(v);
    }
  }
  const int live = __syncthreads_or(nz);
  if (threadIdx.x == 0 && kmask) kmask[static_cast<int64_t>(tile) * hsd::mask_row_bytes(kmax) + grp] = live ? 1 : 0;
}

// y[t, o] = sum_{p = 0..topk} part[t*(topk+1) + p, o] (+ resid), fixed order.
template <typename YT>
__global__ void __launch_bounds__(256) partial_reduce_kernel(const float* __restrict__ part, const void* resid,
                                                     void* y, int T, int D, int topk, int nparts) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= static_cast<int64_t>(T) * D) return;
  const int64_t t = i / D, o = i - t * D;
  const float* p = part + t * (topk + 1) * static_cast<int64_t>(D) + o;
  float acc = 0.f;
  for (int k = 0; k < nparts; ++k) acc += p[static_cast<int64_t>(k) * D];   // (no shared row when FS == 0)
  if (resid) acc += hsd::to_f32<YT>(reinterpret_cast<const YT*>(resid)[i]);
  reinterpret_cast<YT*>(y)[i] = hsd::from_f32<YT>(acc);
}

}  // namespace

namespace hsd {

int prefill_tile_counts(int T, int topk, int E, int tt, int* nt_routed, int* nt_shared) {
  if (T < 1 || topk < 1 || E < 1 || tt < 1)
    return set_error(HSD_ERR_SHAPE, "prefill tiles: need T, topk, E, tt >= 1");
  // the reference's fixed bound T*topk//tt + E (hsd/prefill.py:266). It always holds: with
  // T*topk = q*tt + r (r < tt), sum_e ceil(c_e/tt) <= (q*tt + r + E*(tt-1))/tt
  // = q + E + (r - E)/tt < q + E + 1.
  long long r = static_cast<long long>(T) * topk / tt + E;
  long long s = (static_cast<long long>(T) + tt - 1) / tt;
  if (r + s > (1ll << 28)) return set_error(HSD_ERR_SHAPE, "prefill tiles: too many tiles");
  *nt_routed = static_cast<int>(r);
  *nt_shared = static_cast<int>(s);
  return HSD_OK;
}

int launch_build_tiles(const int32_t* sel, int T, int topk, int E, int tt, int nt_routed, int nt_shared,
                       int T_shared, const int* nslots_dev, int32_t* tile_e, int32_t* tile_slot, cudaStream_t st) {
  if (E > kMaxExperts) return set_error(HSD_ERR_SHAPE, "prefill build_tiles: E > %d", kMaxExperts);
  if (static_cast<long long>(T) * topk > (1ll << 30)) return set_error(HSD_ERR_SHAPE, "prefill build_tiles: too many slots");
  build_tiles_kernel<<<1, kTileThreads, 0, st>>>(sel, T, topk, E, tt, nt_routed, nt_shared, T_shared, nslots_dev,
                                                 tile_e, tile_slot);
  return check_launch("prefill build_tiles");
}

int launch_gather(const void* h, int h_dtype, const int32_t* tile_e, const int32_t* tile_slot, int NT,
                  int tt, int F, int FS, int topk, int E, int kmax, __half* hc, uint8_t* kmask, cudaStream_t st,
                  const void* hs, int64_t hs_stride, int64_t h_stride) {
  const dim3 grid(static_cast<unsigned>(kmax / 64), static_cast<unsigned>(NT));
  if (h_stride <= 0) h_stride = static_cast<int64_t>(topk) * F + FS;
  const int esz = h_dtype == HSD_F32 ? 4 : 2;
  if (!hs) {
    hs = static_cast<const unsigned char*>(h) + static_cast<int64_t>(topk) * F * esz;
    hs_stride = static_cast<int64_t>(topk) * F + FS;
  }
  switch (h_dtype) {
    case HSD_F32:
      gather_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(h), h_stride, tile_e, tile_slot, tt, F, FS,
                                                 topk, E, kmax, hc, kmask, static_cast<const float*>(hs), hs_stride);
      break;
    case HSD_F16:
      gather_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(h), h_stride, tile_e, tile_slot, tt, F,
                                                  FS, topk, E, kmax, hc, kmask, static_cast<const __half*>(hs),
                                                  hs_stride);
      break;
    case HSD_BF16:
      gather_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(h), h_stride, tile_e,
                                                         tile_slot, tt, F, FS, topk, E, kmax, hc, kmask,
                                                         static_cast<const __nv_bfloat16*>(hs), hs_stride);
      break;
    default: return set_error(HSD_ERR_DTYPE, "prefill gather: h_dtype %d", h_dtype);
  }
  return check_launch("prefill gather");
}

int launch_reduce(const float* part, const void* resid, void* y, int y_dtype, int T, int D, int topk,
                  int nparts, cudaStream_t st) {
  const int64_t n = static_cast<int64_t>(T) * D;
  const unsigned grid = static_cast<unsigned>((n + 255) / 256);
  switch (y_dtype) {
    case HSD_F32: partial_reduce_kernel<float><<<grid, 256, 0, st>>>(part, resid, y, T, D, topk, nparts); break;
    case HSD_F16: partial_reduce_kernel<__half><<<grid, 256, 0, st>>>(part, resid, y, T, D, topk, nparts); break;
    case HSD_BF16: partial_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(part, resid, y, T, D, topk, nparts); break;
    default: return set_error(HSD_ERR_DTYPE, "prefill reduce: y_dtype %d", y_dtype);
  }
  return check_launch("prefill reduce");
}

}  // namespace hsd

// ---- C ABI -------------------------------------------------------------------------------

extern "C" int hsd_prefill_num_tiles(int T, int topk, int E, int tt, int* nt_routed, int* nt_shared) {
  if (!nt_routed || !nt_shared) return hsd::set_error(HSD_ERR_ARG, "hsd_prefill_num_tiles: null output");
  return hsd::prefill_tile_counts(T, topk, E, tt, nt_routed, nt_shared);
}

extern "C" int hsd_prefill_build_tiles(const int32_t* sel, int T, int topk, int E, int tt, int32_t* tile_e,
                                       int32_t* tile_slot, void* stream) {
  if (!sel || !tile_e || !tile_slot) return hsd::set_error(HSD_ERR_ARG, "hsd_prefill_build_tiles: null pointer");
  int nr = 0, ns = 0;
  int rc = hsd::prefill_tile_counts(T, topk, E, tt, &nr, &ns);
  if (rc) return rc;
  return hsd::launch_build_tiles(sel, T, topk, E, tt, nr, ns, T, nullptr, tile_e, tile_slot, hsd::as_stream(stream));
}

extern "C" int hsd_prefill_build_union(const void* h, int h_dtype, const int32_t* tile_e, const int32_t* tile_slot,
                                       int NT, int tt, int F, int FS, int topk, int E, int umax, int32_t* ulist,
                                       int32_t* ucount, void* stream) {
  if (!h || !tile_e || !tile_slot || !ulist || !ucount)
    return hsd::set_error(HSD_ERR_ARG, "hsd_prefill_build_union: null pointer");
  if (NT < 1 || tt < 1 || tt > 1024 || F < 1 || FS < 1 || topk < 1 || E < 1 || umax < FS || umax < F)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_prefill_build_union: bad shape (tt <= 1024, umax >= F, FS)");
  cudaStream_t st = hsd::as_stream(stream);
  switch (h_dtype) {
    case HSD_F32:
      build_union_kernel<float><<<NT, 256, 0, st>>>(static_cast<const float*>(h), tile_e, tile_slot, tt, F, FS, topk,
                                                     E, umax, ulist, ucount);
      break;
    case HSD_F16:
      build_union_kernel<__half><<<NT, 256, 0, st>>>(static_cast<const __half*>(h), tile_e, tile_slot, tt, F, FS,
                                                      topk, E, umax, ulist, ucount);
      break;
    case HSD_BF16:
      build_union_kernel<__nv_bfloat16><<<NT, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(h), tile_e, tile_slot,
                                                             tt, F, FS, topk, E, umax, ulist, ucount);
      break;
    default: return hsd::set_error(HSD_ERR_DTYPE, "hsd_prefill_build_union: h_dtype %d", h_dtype);
  }
  return hsd::check_launch("hsd_prefill_build_union");
}

namespace {
struct PrefillWorkspace {
  size_t km_off, hc_off, hc_bytes, part_off, part_bytes, total;
};
int prefill_workspace(int T, int D, int F, int FS, int topk, int E, PrefillWorkspace* w) {
  int nr = 0, ns = 0;
  int rc = hsd::prefill_tile_counts(T, topk, E, hsd::kPrefillTile, &nr, &ns);
  if (rc) return rc;
  const size_t kmax = static_cast<size_t>(F > FS ? F : FS);
  w->km_off = 0;
  w->hc_off = (static_cast<size_t>(nr + ns) * hsd::mask_row_bytes(static_cast<int>(kmax)) + 255) / 256 * 256;
  w->hc_bytes = static_cast<size_t>(nr + ns) * hsd::kPrefillTile * kmax * 2;
  w->part_off = (w->hc_off + w->hc_bytes + 255) / 256 * 256;
  w->part_bytes = static_cast<size_t>(T) * (topk + 1) * D * 4;
  w->total = w->part_off + w->part_bytes;
  return HSD_OK;
}
}  // namespace

extern "C" int hsd_prefill_workspace_bytes(int T, int D, int F, int FS, int topk, int E, size_t* bytes) {
  if (!bytes) return hsd::set_error(HSD_ERR_ARG, "hsd_prefill_workspace_bytes: null output");
  PrefillWorkspace w;
  int rc = prefill_workspace(T, D, F, FS, topk, E, &w);
  if (rc) return rc;
  *bytes = w.total;
  return HSD_OK;
}

extern "C" int hsd_sparse_down_prefill(const void* h, int h_dtype, const float* gains, const int32_t* tile_e,
                                       const int32_t* tile_slot, int NT, const uint32_t* pw, const void* ps,
                                       const void* pb, int s_dtype, const uint32_t* spw, const void* sps,
                                       const void* spb, const void* resid, void* y, int y_dtype, int T, int D, int F,
                                       int FS, int topk, int E, void* workspace, size_t workspace_bytes,
                                       void* stream) {
  if (!h || !gains || !tile_e || !tile_slot || !pw || !ps || !pb || !y || !workspace ||
      (FS > 0 && (!spw || !sps || !spb)))
    return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_prefill: null pointer");
  if (T < 1 || D < 192 || D % 192 != 0 || F < 64 || F % 64 != 0 || FS < 0 || FS % 64 != 0 || topk < 1 || E < 1)
    return hsd::set_error(HSD_ERR_SHAPE,
                          "hsd_sparse_down_prefill: need D %% 192 == 0, F %% 64 == 0, FS %% 64 == 0 "
                          "(got T=%d D=%d F=%d FS=%d topk=%d E=%d)", T, D, F, FS, topk, E);
  int nr = 0, ns = 0;
  int rc = hsd::prefill_tile_counts(T, topk, E, hsd::kPrefillTile, &nr, &ns);
  if (rc) return rc;
  if (NT != nr + ns)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_sparse_down_prefill: tiles must be built with tt = %d (NT %d, expected %d)",
                          hsd::kPrefillTile, NT, nr + ns);
  PrefillWorkspace w;
  rc = prefill_workspace(T, D, F, FS, topk, E, &w);
  if (rc) return rc;
  if (workspace_bytes < w.total)
    return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_prefill: workspace %zu bytes, need %zu", workspace_bytes, w.total);
  const void* p16[] = {pw, ps, pb, spw, sps, spb, workspace};
  for (const void* q : p16)
    if (!hsd::aligned(q, 16))
      return hsd::set_error(HSD_ERR_ALIGN, "hsd_sparse_down_prefill: weights and workspace must be 16-byte aligned");
  cudaStream_t st = hsd::as_stream(stream);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  uint8_t* kmask = ws + w.km_off;
  __half* hc = reinterpret_cast<__half*>(ws + w.hc_off);
  float* part = reinterpret_cast<float*>(ws + w.part_off);
  const int kmax = F > FS ? F : FS;
  rc = hsd::launch_gather(h, h_dtype, tile_e, tile_slot, NT, hsd::kPrefillTile, F, FS, topk, E, kmax, hc, kmask, st);
  if (rc) return rc;
  rc = hsd::launch_prefill_gemm(hc, kmax, tile_e, tile_slot, NT, kmask, gains, pw, ps, pb, s_dtype, spw, sps, spb,
                                part, T, D, F, FS, topk, E, st);
  if (rc) return rc;
  return hsd::launch_reduce(part, resid, y, y_dtype, T, D, topk, topk + (FS > 0 ? 1 : 0), st);
}
