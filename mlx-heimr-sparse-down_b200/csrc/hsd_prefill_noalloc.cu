// Allocation-free variant of the prefill down projection, for callers that cannot call
// cudaMalloc: code running while a CUDA graph is being captured without a memory pool,
// runtimes that own every device allocation themselves, or hosts that must not grow device
// memory after start-up. It computes exactly what hsd_sparse_down_prefill computes, but
// keeps its scratch (the compacted tile order, the live-K-tile masks, the gathered fp16 A
// rows and the fp32 partial rows) in one file-scope device array of kNoAllocScratchBytes instead of a
// caller workspace. Every GPU that loads this library holds that array until the process
// exits. Calls share the array, so calls whose work overlaps on the GPU (two streams, or
// two host threads) race; calls ordered on one stream do not.
#include <mutex>

#include "hsd_common.cuh"
#include "hsd_prefill.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;   // 64 MiB per device
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on each device (host code only sees a stand-in
// for the symbol, never its device address), looked up once per device.
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return hsd::check_cuda(e, "hsd_sparse_down_prefill_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_prefill_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);   // with `dev` current
    if (e != cudaSuccess) return hsd::check_cuda(e, "hsd_sparse_down_prefill_noalloc: cudaGetSymbolAddress");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return HSD_OK;
}

// Copies the non-empty tiles of (tile_e, tile_slot), in order, into the first entries of
// (tile_e_c, tile_slot_c) of capacity NC and marks the rest empty (-1). One CTA; NT is a
// few hundred tiles at most for the chunk sizes the scratch admits.
__global__ void __launch_bounds__(1024) compact_tiles_kernel(const int32_t* __restrict__ tile_e,
                                                             const int32_t* __restrict__ tile_slot, int NT, int tt,
                                                             int NC, int32_t* __restrict__ tile_e_c,
                                                             int32_t* __restrict__ tile_slot_c) {
  __shared__ int pos[4096];
  if (threadIdx.x == 0) {
    int n = 0;
    for (int t = 0; t < NT; ++t) pos[t] = (tile_e[t] >= 0) ? n++ : -1;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < NC; i += blockDim.x) tile_e_c[i] = -1;
  for (int i = threadIdx.x; i < NC * tt; i += blockDim.x) tile_slot_c[i] = -1;
  __syncthreads();
  for (int t = threadIdx.x; t < NT; t += blockDim.x) {
    const int c = pos[t];
    if (c >= 0 && c < NC) tile_e_c[c] = tile_e[t];
  }
  for (int i = threadIdx.x; i < NT * tt; i += blockDim.x) {
    const int c = pos[i / tt];
    if (c >= 0 && c < NC) tile_slot_c[c * tt + i % tt] = tile_slot[i];
  }
}

struct NoAllocLayout {
  int NC;                 // capacity of the compacted tile order
  size_t te_off, ts_off, km_off, hc_off, part_off, total;
};

// Non-empty tiles are at most: every full tile of slots plus one partial tile per expert
// that has slots (at most min(E, T*topk)), plus the shared expert's tiles.
int noalloc_layout(int T, int D, int F, int FS, int topk, int E, int NT, NoAllocLayout* L) {
  int nr = 0, ns = 0;
  int rc = hsd::prefill_tile_counts(T, topk, E, hsd::kPrefillTile, &nr, &ns);
  if (rc) return rc;
  const long long slots = static_cast<long long>(T) * topk;
  long long routed = slots / hsd::kPrefillTile + (E < slots ? E : slots);
  if (routed > nr) routed = nr;
  L->NC = static_cast<int>(routed + ns);
  const size_t kmax = static_cast<size_t>(F > FS ? F : FS);
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  L->te_off = 0;
  L->ts_off = up(L->te_off + sizeof(int32_t) * L->NC);
  L->km_off = up(L->ts_off + sizeof(int32_t) * static_cast<size_t>(L->NC) * hsd::kPrefillTile);
  L->hc_off = up(L->km_off + static_cast<size_t>(L->NC) * hsd::mask_row_bytes(static_cast<int>(kmax)));
  L->part_off = up(L->hc_off + static_cast<size_t>(L->NC) * hsd::kPrefillTile * kmax * 2);
  L->total = L->part_off + static_cast<size_t>(T) * (topk + 1) * D * 4;
  if (NT != nr + ns)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_sparse_down_prefill_noalloc: tiles must be built with tt = %d",
                          hsd::kPrefillTile);
  if (NT > 4096) return hsd::set_error(HSD_ERR_SHAPE, "hsd_sparse_down_prefill_noalloc: more than 4096 tiles");
  return HSD_OK;
}

}  // namespace

// Also looks up the array's address on the current device, so a caller can do the one-time
// set-up without inputs (before a stream capture, for instance).
extern "C" int hsd_prefill_noalloc_max_bytes(size_t* bytes) {
  if (!bytes) return hsd::set_error(HSD_ERR_ARG, "hsd_prefill_noalloc_max_bytes: null output");
  *bytes = kNoAllocScratchBytes;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();                          // no device here: the size alone is the answer
    return HSD_OK;
  }
  void* base = nullptr;
  return scratch_address(&base);
}

extern "C" int hsd_sparse_down_prefill_noalloc(const void* h, int h_dtype, const float* gains,
                                               const int32_t* tile_e, const int32_t* tile_slot, int NT,
                                               const uint32_t* pw, const void* ps, const void* pb, int s_dtype,
                                               const uint32_t* spw, const void* sps, const void* spb,
                                               const void* resid, void* y, int y_dtype, int T, int D, int F, int FS,
                                               int topk, int E, void* stream) {
  if (!h || !gains || !tile_e || !tile_slot || !pw || !ps || !pb || !y || (FS > 0 && (!spw || !sps || !spb)))
    return hsd::set_error(HSD_ERR_ARG, "hsd_sparse_down_prefill_noalloc: null pointer");
  if (T < 1 || D < 192 || D % 192 != 0 || F < 64 || F % 64 != 0 || FS < 0 || FS % 64 != 0 || topk < 1 || E < 1)
    return hsd::set_error(HSD_ERR_SHAPE,
                          "hsd_sparse_down_prefill_noalloc: need D %% 192 == 0, F %% 64 == 0, FS %% 64 == 0 "
                          "(got T=%d D=%d F=%d FS=%d topk=%d E=%d)", T, D, F, FS, topk, E);
  NoAllocLayout L;
  int rc = noalloc_layout(T, D, F, FS, topk, E, NT, &L);
  if (rc) return rc;
  if (L.total > kNoAllocScratchBytes)
    return hsd::set_error(HSD_ERR_SHAPE,
                          "hsd_sparse_down_prefill_noalloc: this call needs %zu bytes of scratch, more than the "
                          "library's fixed %zu (T=%d D=%d F=%d FS=%d topk=%d E=%d); use hsd_sparse_down_prefill "
                          "with a caller workspace or a smaller chunk",
                          L.total, kNoAllocScratchBytes, T, D, F, FS, topk, E);
  const void* p16[] = {pw, ps, pb, spw, sps, spb};
  for (const void* q : p16)
    if (!hsd::aligned(q, 16))
      return hsd::set_error(HSD_ERR_ALIGN, "hsd_sparse_down_prefill_noalloc: weights must be 16-byte aligned");
  void* base = nullptr;
  rc = scratch_address(&base);
  if (rc) return rc;
  unsigned char* ws = static_cast<unsigned char*>(base);
  int32_t* te_c = reinterpret_cast<int32_t*>(ws + L.te_off);
  int32_t* ts_c = reinterpret_cast<int32_t*>(ws + L.ts_off);
  uint8_t* kmask = ws + L.km_off;
  __half* hc = reinterpret_cast<__half*>(ws + L.hc_off);
  float* part = reinterpret_cast<float*>(ws + L.part_off);
  cudaStream_t st = hsd::as_stream(stream);
  // every scratch byte the later kernels read is written first in this call: the compacted
  // tile order in full, the live-K-tile mask bytes and the A rows of every non-empty tile
  // (zero rows for padding slots), and every partial row of every token
  compact_tiles_kernel<<<1, 1024, 0, st>>>(tile_e, tile_slot, NT, hsd::kPrefillTile, L.NC, te_c, ts_c);
  rc = hsd::check_launch("hsd_sparse_down_prefill_noalloc: compact");
  if (rc) return rc;
  const int kmax = F > FS ? F : FS;
  rc = hsd::launch_gather(h, h_dtype, te_c, ts_c, L.NC, hsd::kPrefillTile, F, FS, topk, E, kmax, hc, kmask, st);
  if (rc) return rc;
  rc = hsd::launch_prefill_gemm(hc, kmax, te_c, ts_c, L.NC, kmask, gains, pw, ps, pb, s_dtype, spw, sps, spb, part, T, D, F,
                                FS, topk, E, st);
  if (rc) return rc;
  return hsd::launch_reduce(part, resid, y, y_dtype, T, D, topk, topk + (FS > 0 ? 1 : 0), st);
}
