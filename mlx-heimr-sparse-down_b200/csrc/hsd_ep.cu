// Expert parallelism over the GPUs of one box (a multi-GPU form of hsd/decode.py's sparse_down
// and hsd/prefill.py's sparse_down_prefill; the reference runs on one Apple GPU).
//
// Routed expert e lives on rank e % G (round robin) unless a placement table says otherwise
// (emap[e] = owner << 16 | local id; hot experts replicated on every rank map to the home rank
// itself, so their slots never leave it), the shared expert is replicated, tokens stay on their
// home rank. Every rank owns an INBOX: device memory allocated with
// hsd_ep_alloc, mapped into every other rank's process (CUDA IPC), which the other ranks write
// with plain stores over NVLink -- no collective library, no multicast, no host round trip:
//
//   header     cnt_flag[s]  epoch of source s's count row        (st.release.sys by s)
//              arr_rows     scatter CTAs of all sources finished  (red.release.sys by the sources)
//              arr_y        owners finished writing partial rows  (red.release.sys by the owners)
//              epoch        this rank's call counter              (this rank only)
//              cnt[s][d]    slots source s sends to rank d        (every source writes its row everywhere)
//   h_in       [R][F]       the slots this rank owns: h rows      (R = G * S receive capacity,
//   sel_in     [R]          ... local expert id                    S = max_tokens * topk)
//   g_in       [R][2]       ... routing gain; [t][1]: this rank's token t's shared-expert gain
//   ret_in     [R]          ... source rank * S + source slot
//   ysl        [S+T][D] f32 this rank's slots' partial rows, written by their owners, then its
//                           tokens' shared-expert rows (T = max_tokens), written by itself
//
// One call, all on the caller's stream (every rank makes the same calls in the same order):
//   hsd_ep_dispatch  route: per-slot destination and stable position, the count row to every
//                    rank, then (all CTAs, after the G count rows of this epoch are in) each
//                    slot's h row, id, gain and return address stored into its owner's inbox at
//                    base(src -> owner) + position; arrivals counted on the owner
//   hsd_ep_expert    wait for every source's scatter CTAs; the received rows' return addresses;
//                    the expert-sorted tile order over the R received rows (count read on the
//                    device) followed by the shared expert's tiles of this rank's own tokens;
//                    ONE tcgen05 grouped GEMM over both, whose epilogue stores each fp32 partial
//                    row, times its gain, straight into its home rank's ysl row (over NVLink;
//                    the shared rows into this rank's own); then one arrival on every rank
//   hsd_ep_combine   wait for the G owners; y[b] = sum_k ysl[b*topk + k] + ysl[S + b], fixed
//                    order
// Nothing is read back to the host, so the call can be captured in a CUDA graph. The counters
// are cumulative (compared modulo 2^32), so no buffer is ever reset. A rank reaches call n+1
// only after its combine of call n has seen every owner's arrival, which every owner sends
// after it has read everything call n put in its inbox: one set of buffers serves every call.
// Every wait is bounded (timeout_s of %globaltimer): running out sets HSD_ERR_TIMEOUT in the
// status word and the kernel goes on without the data (the call's output is then unspecified
// and the ranks must rebuild their inboxes); every index read from another rank is
// range-checked before it addresses memory.
#include <cstring>

#include "hsd_common.cuh"
#include "hsd_prefill.cuh"

HSD_DEFINE_STATUS(ep)

namespace {

constexpr int kMaxWorld = 16;
constexpr int kScatterCTAs = 128;   // fixed: an owner's arrival target counts every source's CTAs
constexpr int kScatterThreads = 256;
constexpr int kRouteThreads = 1024;
constexpr int kCombineThreads = 256;

constexpr size_t kOffCntFlag = 0;    // uint32 [kMaxWorld]
constexpr size_t kOffArrRows = 128;  // uint32
constexpr size_t kOffArrY = 256;     // uint32
constexpr size_t kOffEpoch = 384;    // uint32
constexpr size_t kOffCnt = 1024;     // int32 [kMaxWorld][kMaxWorld]
constexpr size_t kHdrBytes = 4096;

constexpr size_t up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct EpLayout {
  int G, S, R, T, F, FS, D, E_local, NT_routed, NT, kmax, mrb;
  // inbox offsets
  size_t h_in, sel_in, g_in, ret_in, ysl, inbox_bytes;
  // workspace offsets
  size_t w_peers, w_misc, w_pos, w_te, w_ts, w_km, w_hc, w_rowdst, ws_bytes;
};

// n_local: the routed experts this rank holds (<= 0: E / world, the round-robin share); only
// the private workspace depends on it, the inbox layout is the same on every rank.
int ep_layout(int world, int max_tokens, int topk, int F, int FS, int D, int E, int n_local, EpLayout* L) {
  if (world < 1 || world > kMaxWorld)
    return hsd::set_error(HSD_ERR_SHAPE, "ep: world %d outside 1..%d", world, kMaxWorld);
  if (max_tokens < 1 || topk < 1 || F < 64 || F % 64 != 0 || FS < 0 || FS % 64 != 0 || D < 192 || D % 192 != 0 ||
      E < 1 || E % world != 0)
    return hsd::set_error(HSD_ERR_SHAPE,
                          "ep: need max_tokens, topk >= 1, F and FS %% 64 == 0, D %% 192 == 0, E %% world == 0 "
                          "(max_tokens=%d topk=%d F=%d FS=%d D=%d E=%d world=%d)", max_tokens, topk, F, FS, D, E,
                          world);
  const long long S = static_cast<long long>(max_tokens) * topk;
  if (S >= (1ll << 24) || S * world >= (1ll << 27))
    return hsd::set_error(HSD_ERR_SHAPE, "ep: max_tokens * topk * world too large (%lld slots)", S * world);
  if (n_local <= 0) n_local = E / world;
  if (n_local > 256 || n_local > E) return hsd::set_error(HSD_ERR_SHAPE, "ep: %d local experts (at most 256 and E)", n_local);
  L->G = world;
  L->S = static_cast<int>(S);
  L->R = static_cast<int>(S * world);
  L->T = max_tokens;
  L->F = F;
  L->FS = FS;
  L->D = D;
  L->E_local = n_local;
  int nr = 0, ns = 0;
  int rc = hsd::prefill_tile_counts(L->R, 1, L->E_local, hsd::kPrefillTile, &nr, &ns);
  if (rc) return rc;
  L->NT_routed = nr;                                 // then the shared expert's tiles of this rank's tokens
  L->NT = nr + (FS > 0 ? (max_tokens + hsd::kPrefillTile - 1) / hsd::kPrefillTile : 0);
  L->kmax = F > FS ? F : FS;
  L->mrb = hsd::mask_row_bytes(L->kmax);
  const size_t R = static_cast<size_t>(L->R);
  L->h_in = kHdrBytes;
  L->sel_in = up(L->h_in + R * F * 2, 256);
  L->g_in = up(L->sel_in + R * 4, 256);
  L->ret_in = up(L->g_in + R * 8, 256);
  L->ysl = up(L->ret_in + R * 4, 256);
  L->inbox_bytes = L->ysl + (static_cast<size_t>(L->S) + max_tokens) * D * 4;
  const size_t NT = static_cast<size_t>(L->NT);
  L->w_peers = 0;
  L->w_misc = 256;
  L->w_pos = 512;
  L->w_te = up(L->w_pos + static_cast<size_t>(L->S) * 4, 256);
  L->w_ts = up(L->w_te + NT * 4, 256);
  L->w_km = up(L->w_ts + NT * hsd::kPrefillTile * 4, 256);
  L->w_hc = up(L->w_km + NT * L->mrb, 256);
  L->w_rowdst = up(L->w_hc + NT * hsd::kPrefillTile * L->kmax * 2, 256);
  L->ws_bytes = L->w_rowdst + R * 8;
  return HSD_OK;
}

// ---- memory-model helpers (system scope: the other side is another GPU)
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits until *p has reached `target` (modulo 2^32); false after timeout_ns.
__device__ bool wait_reached(const uint32_t* p, uint32_t target, uint64_t timeout_ns) {
  if (static_cast<int32_t>(ld_acquire_sys(p) - target) >= 0) return true;
  const uint64_t t0 = now_ns();
  while (static_cast<int32_t>(ld_acquire_sys(p) - target) < 0) {
    if (now_ns() - t0 > timeout_ns) return false;
    __nanosleep(256);
  }
  return true;
}

__device__ __forceinline__ unsigned char* inbox(const uint64_t* peers, int r) {
  return reinterpret_cast<unsigned char*>(peers[r]);
}
__device__ __forceinline__ uint32_t own_epoch(const uint64_t* peers, int rank) {
  return *reinterpret_cast<volatile const uint32_t*>(inbox(peers, rank) + kOffEpoch);
}

struct InboxOffsets {
  unsigned long long h_in, sel_in, g_in, ret_in, ysl;
};

// ---- route (one CTA): the call's epoch, each slot's destination (expert % G) and stable
//      position among the slots going there (ascending slot order), and this rank's count row
//      written into every rank's inbox, then published with the epoch.
__global__ void __launch_bounds__(kRouteThreads) ep_route_kernel(const uint64_t* __restrict__ peers, int rank, int G,
                                                                 const int32_t* __restrict__ sel, int nslots, int E,
                                                                 const int32_t* __restrict__ emap,
                                                                 int32_t* __restrict__ pos) {
  __shared__ int running[kMaxWorld];
  __shared__ int tab[kRouteThreads / 32][kMaxWorld];
  __shared__ uint32_t epoch_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) epoch_s = own_epoch(peers, rank) + 1u;
  if (tid < kMaxWorld) running[tid] = 0;
  __syncthreads();
  for (int c0 = 0; c0 < nslots; c0 += kRouteThreads) {
    const int j = c0 + tid;
    int d = -1;
    if (j < nslots) {
      const int e = sel[j];
      const int o = (e >= 0 && e < E) ? (emap ? (emap[e] >> 16) : e % G) : -1;
      if (o >= 0 && o < G) {
        d = o;
      } else {
        hsd_flag_ep(HSD_ERR_INDEX);   // kept home without an expert: the owner drops it
        d = rank;
      }
    }
    int below = 0;
    for (int q = 0; q < G; ++q) {
      const unsigned m = __ballot_sync(0xffffffffu, d == q);
      if (lane == 0) tab[warp][q] = __popc(m);
      if (d == q) below = __popc(m & ((1u << lane) - 1u));
    }
    __syncthreads();
    if (tid < G) {                                  // exclusive scan over the warps, after the earlier chunks
      int acc = running[tid];
      for (int w = 0; w < kRouteThreads / 32; ++w) {
        const int v = tab[w][tid];
        tab[w][tid] = acc;
        acc += v;
      }
      running[tid] = acc;
    }
    __syncthreads();
    if (d >= 0) pos[j] = (tab[warp][d] + below) | (d << 24);
    __syncthreads();
  }
  if (tid == 0) {
    const uint32_t epoch = epoch_s;
    for (int q = 0; q < G; ++q) {
      int32_t* row = reinterpret_cast<int32_t*>(inbox(peers, q) + kOffCnt) + rank * kMaxWorld;
      for (int d = 0; d < G; ++d) row[d] = running[d];
    }
    __threadfence_system();
    for (int q = 0; q < G; ++q)
      st_release_sys(reinterpret_cast<uint32_t*>(inbox(peers, q) + kOffCntFlag) + rank, epoch);
    *reinterpret_cast<volatile uint32_t*>(inbox(peers, rank) + kOffEpoch) = epoch;
  }
}

// ---- scatter (kScatterCTAs CTAs): once the G count rows of this epoch are in, each slot's h
//      row (16-byte pieces, one warp a slot), local expert id, gain and return address go to
//      row base(rank -> owner) + position of the owner's inbox; this rank's tokens'
//      shared-expert gains go to its own inbox (g_in[t][1]); then every CTA counts one arrival
//      on every rank.
__global__ void __launch_bounds__(kScatterThreads) ep_scatter_kernel(const uint64_t* __restrict__ peers, int rank,
                                                                     int G, int S, const unsigned char* __restrict__ hcat,
                                                                     const int32_t* __restrict__ sel,
                                                                     const float* __restrict__ gains,
                                                                     const int32_t* __restrict__ pos, int nslots,
                                                                     int topk, int F, int FS, int E,
                                                                     const int32_t* __restrict__ emap, InboxOffsets off,
                                                                     unsigned long long timeout_ns) {
  const int NR = topk * F + FS;
  __shared__ int base[kMaxWorld];
  __shared__ int ok_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    const uint32_t epoch = own_epoch(peers, rank);
    const uint32_t* flags = reinterpret_cast<const uint32_t*>(inbox(peers, rank) + kOffCntFlag);
    bool ok = true;
    for (int s = 0; s < G && ok; ++s) ok = wait_reached(flags + s, epoch, timeout_ns);
    if (!ok) hsd_flag_ep(HSD_ERR_TIMEOUT);
    ok_s = ok ? 1 : 0;
  }
  __syncthreads();
  if (ok_s && tid < G) {
    const volatile int32_t* cnt = reinterpret_cast<const volatile int32_t*>(inbox(peers, rank) + kOffCnt);
    int b = 0;
    for (int s = 0; s < rank; ++s) b += cnt[s * kMaxWorld + tid];
    base[tid] = b;
  }
  __syncthreads();
  if (ok_s) {
    const int row_bytes = F * 2;
    for (int j = blockIdx.x * (kScatterThreads / 32) + warp; j < nslots; j += gridDim.x * (kScatterThreads / 32)) {
      const int p = pos[j];
      const int d = p >> 24, row = base[d] + (p & 0xFFFFFF);
      if (d >= G || row >= G * S) continue;        // (cannot happen with this epoch's counts)
      unsigned char* dst = inbox(peers, d);
      const int b = j / topk, k = j - b * topk;
      const uint4* src = reinterpret_cast<const uint4*>(hcat + (static_cast<int64_t>(b) * NR + static_cast<int64_t>(k) * F) * 2);
      uint4* dh = reinterpret_cast<uint4*>(dst + off.h_in + static_cast<int64_t>(row) * row_bytes);
      for (int i = lane; i < row_bytes / 16; i += 32) dh[i] = hsd::ldg_nc_v4(src + i);
      if (lane == 0) {
        const int e = sel[j];
        reinterpret_cast<int32_t*>(dst + off.sel_in)[row] = (e >= 0 && e < E) ? (emap ? (emap[e] & 0xFFFF) : e / G) : -1;
        reinterpret_cast<float*>(dst + off.g_in)[2 * static_cast<int64_t>(row)] =
            gains[static_cast<int64_t>(b) * (topk + 1) + k];
        reinterpret_cast<int32_t*>(dst + off.ret_in)[row] = rank * S + j;
      }
    }
  }
  if (FS > 0) {                                    // (g_in[t][1] of a received row is never read)
    float* own_g = reinterpret_cast<float*>(inbox(peers, rank) + off.g_in);
    for (int t = blockIdx.x * kScatterThreads + tid; t < nslots / topk; t += gridDim.x * kScatterThreads)
      own_g[2 * static_cast<int64_t>(t) + 1] = gains[static_cast<int64_t>(t) * (topk + 1) + topk];
  }
  __threadfence_system();
  __syncthreads();
  if (tid < G) red_add_release_sys(reinterpret_cast<uint32_t*>(inbox(peers, tid) + kOffArrRows), 1u);
}

// ---- receive (one CTA): wait for every source's scatter CTAs, the received row count
//      (written for the tile builder) and each received row's output address: the source's
//      ysl row of the slot (checked against the world and the slot capacity; null drops it).
__global__ void __launch_bounds__(1024) ep_recv_kernel(const uint64_t* __restrict__ peers, int rank, int G, int S,
                                                       int D, InboxOffsets off, int* __restrict__ nrecv,
                                                       float** __restrict__ row_dst, unsigned long long timeout_ns) {
  __shared__ int R_s;
  const int tid = threadIdx.x;
  if (tid == 0) {
    const uint32_t epoch = own_epoch(peers, rank);
    const bool ok = wait_reached(reinterpret_cast<const uint32_t*>(inbox(peers, rank) + kOffArrRows),
                                 epoch * static_cast<uint32_t>(G * kScatterCTAs), timeout_ns);
    int R = 0;
    if (ok) {
      const volatile int32_t* cnt = reinterpret_cast<const volatile int32_t*>(inbox(peers, rank) + kOffCnt);
      for (int s = 0; s < G; ++s) R += min(max(static_cast<int>(cnt[s * kMaxWorld + rank]), 0), S);
    } else {
      hsd_flag_ep(HSD_ERR_TIMEOUT);
    }
    R_s = R;
    *nrecv = R;
  }
  __syncthreads();
  const int R = R_s;
  const int32_t* ret = reinterpret_cast<const int32_t*>(inbox(peers, rank) + off.ret_in);
  for (int i = tid; i < R; i += 1024) {
    const int v = ret[i];
    const int sr = v / S, j = v - (v / S) * S;
    row_dst[i] = (v >= 0 && sr < G) ? reinterpret_cast<float*>(inbox(peers, sr) + off.ysl) + static_cast<int64_t>(j) * D
                                    : nullptr;
  }
}

// ---- one arrival on every rank: this rank's partial rows of the call are all stored (the
//      GEMM before it in the stream wrote them).
__global__ void ep_signal_kernel(const uint64_t* __restrict__ peers, int G) {
  __threadfence_system();
  if (static_cast<int>(threadIdx.x) < G)
    red_add_release_sys(reinterpret_cast<uint32_t*>(inbox(peers, threadIdx.x) + kOffArrY), 1u);
}

// ---- combine: wait for the G owners, then y[b] = sum_k ysl[b*topk + k] (+ ysl[S + b], the
//      shared expert's row, when there is one).
__global__ void __launch_bounds__(kCombineThreads) ep_combine_kernel(const uint64_t* __restrict__ peers, int rank, int G,
                                                                     int B, int topk, int S, int shared, int D,
                                                                     InboxOffsets off, float* __restrict__ y,
                                                                     unsigned long long timeout_ns) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    const uint32_t epoch = own_epoch(peers, rank);
    const bool ok = wait_reached(reinterpret_cast<const uint32_t*>(inbox(peers, rank) + kOffArrY),
                                 epoch * static_cast<uint32_t>(G), timeout_ns);
    if (!ok) hsd_flag_ep(HSD_ERR_TIMEOUT);
    ok_s = ok;
  }
  __syncthreads();
  const float4* ysl = reinterpret_cast<const float4*>(inbox(peers, rank) + off.ysl);
  const int D4 = D / 4;
  const int64_t n = static_cast<int64_t>(B) * D4;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kCombineThreads + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * kCombineThreads) {
    const int64_t b = i / D4, o = i - b * D4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < (ok_s ? topk : 0); ++k) {      // (after a timeout: zeros)
      const float4 v = ysl[(b * topk + k) * D4 + o];
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    if (shared && ok_s) {
      const float4 v = ysl[(static_cast<int64_t>(S) + b) * D4 + o];
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    reinterpret_cast<float4*>(y)[i] = a;
  }
}

InboxOffsets offsets_of(const EpLayout& L) {
  InboxOffsets o;
  o.h_in = L.h_in;
  o.sel_in = L.sel_in;
  o.g_in = L.g_in;
  o.ret_in = L.ret_in;
  o.ysl = L.ysl;
  return o;
}

unsigned long long timeout_ns_of(double s) {
  if (!(s > 0.0)) s = 10.0;
  if (s > 3600.0) s = 3600.0;
  return static_cast<unsigned long long>(s * 1e9);
}

int check_rank(int rank, int world, const void* ws) {
  if (!ws) return hsd::set_error(HSD_ERR_ARG, "ep: null workspace");
  if (!hsd::aligned(ws, 256)) return hsd::set_error(HSD_ERR_ALIGN, "ep: workspace must be 256-byte aligned");
  if (rank < 0 || rank >= world) return hsd::set_error(HSD_ERR_ARG, "ep: rank %d outside 0..%d", rank, world - 1);
  return HSD_OK;
}

}  // namespace

// ---- C ABI -------------------------------------------------------------------------------

extern "C" int hsd_ep_buffer_bytes(int world, int max_tokens, int topk, int F, int FS, int D, int E, int n_local,
                                   size_t* inbox_bytes, size_t* workspace_bytes) {
  if (!inbox_bytes || !workspace_bytes) return hsd::set_error(HSD_ERR_ARG, "hsd_ep_buffer_bytes: null output");
  EpLayout L;
  int rc = ep_layout(world, max_tokens, topk, F, FS, D, E, n_local, &L);
  if (rc) return rc;
  *inbox_bytes = L.inbox_bytes;
  *workspace_bytes = L.ws_bytes;
  return HSD_OK;
}

extern "C" int hsd_ep_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return hsd::set_error(HSD_ERR_ARG, "hsd_ep_alloc: null output or zero bytes");
  *ptr = nullptr;
  void* p = nullptr;
  int rc = hsd::check_cuda(cudaMalloc(&p, bytes), "hsd_ep_alloc: cudaMalloc");
  if (rc) return rc;
  rc = hsd::check_cuda(cudaMemset(p, 0, bytes), "hsd_ep_alloc: cudaMemset");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return HSD_OK;
}

extern "C" int hsd_ep_free(void* ptr) {
  if (!ptr) return HSD_OK;
  return hsd::check_cuda(cudaFree(ptr), "hsd_ep_free");
}

extern "C" int hsd_ep_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return hsd::set_error(HSD_ERR_ARG, "hsd_ep_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  int rc = hsd::check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "hsd_ep_ipc_handle");
  if (rc) return rc;
  static_assert(sizeof(h) == HSD_EP_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return HSD_OK;
}

extern "C" int hsd_ep_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return hsd::set_error(HSD_ERR_ARG, "hsd_ep_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  return hsd::check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "hsd_ep_ipc_open");
}

extern "C" int hsd_ep_ipc_close(void* ptr) {
  if (!ptr) return HSD_OK;
  return hsd::check_cuda(cudaIpcCloseMemHandle(ptr), "hsd_ep_ipc_close");
}

extern "C" int hsd_ep_set_peers(void* workspace, const uint64_t* inbox_addrs, int world, void* stream) {
  if (!workspace || !inbox_addrs) return hsd::set_error(HSD_ERR_ARG, "hsd_ep_set_peers: null pointer");
  if (world < 1 || world > kMaxWorld) return hsd::set_error(HSD_ERR_SHAPE, "hsd_ep_set_peers: world %d", world);
  for (int r = 0; r < world; ++r)
    if (inbox_addrs[r] == 0 || inbox_addrs[r] % 256 != 0)
      return hsd::set_error(HSD_ERR_ALIGN, "hsd_ep_set_peers: inbox %d is null or not 256-byte aligned", r);
  cudaStream_t st = hsd::as_stream(stream);
  int rc = hsd::check_cuda(cudaMemcpyAsync(workspace, inbox_addrs, sizeof(uint64_t) * world, cudaMemcpyHostToDevice, st),
                           "hsd_ep_set_peers: copy");
  if (rc) return rc;
  return hsd::check_cuda(cudaStreamSynchronize(st), "hsd_ep_set_peers: synchronize");
}

extern "C" int hsd_ep_dispatch(void* workspace, int rank, int world, int max_tokens, const void* hcat, int h_dtype,
                               const int32_t* sel, const float* gains, int B, int topk, int F, int FS, int D, int E,
                               const int32_t* emap, double timeout_s, void* stream) {
  EpLayout L;
  int rc = ep_layout(world, max_tokens, topk, F, FS, D, E, 0, &L);
  if (rc) return rc;
  if ((rc = check_rank(rank, world, workspace))) return rc;
  if (B < 0 || B > max_tokens)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_ep_dispatch: B=%d outside 0..max_tokens=%d", B, max_tokens);
  if (B > 0 && (!hcat || !sel || !gains)) return hsd::set_error(HSD_ERR_ARG, "hsd_ep_dispatch: null pointer");
  if (h_dtype != HSD_BF16 && h_dtype != HSD_F16)
    return hsd::set_error(HSD_ERR_DTYPE, "hsd_ep_dispatch: h_dtype %d (bf16 or f16)", h_dtype);
  if (hcat && !hsd::aligned(hcat, 16)) return hsd::set_error(HSD_ERR_ALIGN, "hsd_ep_dispatch: hcat must be 16-byte aligned");
  cudaStream_t st = hsd::as_stream(stream);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const uint64_t* peers = reinterpret_cast<const uint64_t*>(ws + L.w_peers);
  int32_t* pos = reinterpret_cast<int32_t*>(ws + L.w_pos);
  ep_route_kernel<<<1, kRouteThreads, 0, st>>>(peers, rank, world, sel, B * topk, E, emap, pos);
  if ((rc = hsd::check_launch("hsd_ep_dispatch: route"))) return rc;
  ep_scatter_kernel<<<kScatterCTAs, kScatterThreads, 0, st>>>(peers, rank, world, L.S,
                                                              static_cast<const unsigned char*>(hcat), sel, gains, pos,
                                                              B * topk, topk, F, FS, E, emap, offsets_of(L),
                                                              timeout_ns_of(timeout_s));
  return hsd::check_launch("hsd_ep_dispatch: scatter");
}

extern "C" int hsd_ep_expert(void* workspace, void* inbox_ptr, int rank, int world, int max_tokens, const void* hcat,
                             int h_dtype, int B, const uint32_t* pw, const void* ps, const void* pb,
                             const uint32_t* spw, const void* sps, const void* spb, int s_dtype, int topk, int F, int FS,
                             int D, int E, int n_local, double timeout_s, void* stream) {
  EpLayout L;
  int rc = ep_layout(world, max_tokens, topk, F, FS, D, E, n_local, &L);
  if (rc) return rc;
  if ((rc = check_rank(rank, world, workspace))) return rc;
  if (B < 0 || B > max_tokens)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_ep_expert: B=%d outside 0..max_tokens=%d", B, max_tokens);
  if (!inbox_ptr || !pw || !ps || !pb || (FS > 0 && (!spw || !sps || !spb)) || (FS > 0 && B > 0 && !hcat))
    return hsd::set_error(HSD_ERR_ARG, "hsd_ep_expert: null pointer");
  if (h_dtype != HSD_BF16 && h_dtype != HSD_F16)
    return hsd::set_error(HSD_ERR_DTYPE, "hsd_ep_expert: h_dtype %d (bf16 or f16)", h_dtype);
  const void* p16[] = {pw, ps, pb, spw, sps, spb, inbox_ptr, hcat};
  for (const void* q : p16)
    if (!hsd::aligned(q, 16))
      return hsd::set_error(HSD_ERR_ALIGN, "hsd_ep_expert: weights, inbox and hcat must be 16-byte aligned");
  cudaStream_t st = hsd::as_stream(stream);
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  unsigned char* ib = static_cast<unsigned char*>(inbox_ptr);
  const uint64_t* peers = reinterpret_cast<const uint64_t*>(ws + L.w_peers);
  int* nrecv = reinterpret_cast<int*>(ws + L.w_misc);
  int32_t* te = reinterpret_cast<int32_t*>(ws + L.w_te);
  int32_t* ts = reinterpret_cast<int32_t*>(ws + L.w_ts);
  uint8_t* km = ws + L.w_km;
  __half* hc = reinterpret_cast<__half*>(ws + L.w_hc);
  float** row_dst = reinterpret_cast<float**>(ws + L.w_rowdst);
  ep_recv_kernel<<<1, 1024, 0, st>>>(peers, rank, world, L.S, D, offsets_of(L), nrecv, row_dst, timeout_ns_of(timeout_s));
  if ((rc = hsd::check_launch("hsd_ep_expert: receive"))) return rc;
  // this call's tiles: the routed ones (fixed count for the capacity), then ceil(B / 128) of
  // the shared expert over this rank's B tokens
  const int ns = (FS > 0) ? (B + hsd::kPrefillTile - 1) / hsd::kPrefillTile : 0;
  const int NT = L.NT_routed + ns;
  const int32_t* sel_in = reinterpret_cast<const int32_t*>(ib + L.sel_in);
  if ((rc = hsd::launch_build_tiles(sel_in, L.R, 1, L.E_local, hsd::kPrefillTile, L.NT_routed, ns, B, nrecv, te, ts, st)))
    return rc;
  const int esz = 2;
  const void* hs = (FS > 0 && hcat) ? static_cast<const unsigned char*>(hcat) + static_cast<int64_t>(topk) * F * esz : nullptr;
  rc = hsd::launch_gather(ib + L.h_in, h_dtype, te, ts, NT, hsd::kPrefillTile, F, FS, 1, L.E_local, L.kmax, hc, km, st,
                          hs ? hs : ib + L.h_in, static_cast<int64_t>(topk) * F + FS, F);
  if (rc) return rc;
  float* shared_out = reinterpret_cast<float*>(ib + L.ysl) + static_cast<int64_t>(L.S) * D;
  rc = hsd::launch_prefill_gemm(hc, L.kmax, te, ts, NT, km, reinterpret_cast<const float*>(ib + L.g_in), pw, ps, pb,
                                s_dtype, spw, sps, spb, nullptr, L.R, D, F, FS, 1, L.E_local, st, row_dst, shared_out);
  if (rc) return rc;
  ep_signal_kernel<<<1, 32, 0, st>>>(peers, world);
  return hsd::check_launch("hsd_ep_expert: signal");
}

extern "C" int hsd_ep_combine(void* workspace, int rank, int world, int max_tokens, float* y, int B, int topk, int F,
                              int FS, int D, int E, double timeout_s, void* stream) {
  EpLayout L;
  int rc = ep_layout(world, max_tokens, topk, F, FS, D, E, 0, &L);
  if (rc) return rc;
  if ((rc = check_rank(rank, world, workspace))) return rc;
  if (B < 0 || B > max_tokens)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_ep_combine: B=%d outside 0..max_tokens=%d", B, max_tokens);
  if (B > 0 && !y) return hsd::set_error(HSD_ERR_ARG, "hsd_ep_combine: null output");
  if (y && !hsd::aligned(y, 16)) return hsd::set_error(HSD_ERR_ALIGN, "hsd_ep_combine: y must be 16-byte aligned");
  cudaStream_t st = hsd::as_stream(stream);
  const uint64_t* peers = reinterpret_cast<const uint64_t*>(static_cast<unsigned char*>(workspace) + L.w_peers);
  // (launched with B = 0 too: its wait orders this rank's next dispatch after every owner's reads)
  const long long n4 = static_cast<long long>(B) * (D / 4);
  long long grid = (n4 + kCombineThreads - 1) / kCombineThreads;
  if (grid < 1) grid = 1;
  if (grid > 4 * 148) grid = 4 * 148;
  ep_combine_kernel<<<static_cast<unsigned>(grid), kCombineThreads, 0, st>>>(peers, rank, world, B, topk, L.S, FS > 0 ? 1 : 0,
                                                                           D, offsets_of(L), y, timeout_ns_of(timeout_s));
  return hsd::check_launch("hsd_ep_combine");
}
