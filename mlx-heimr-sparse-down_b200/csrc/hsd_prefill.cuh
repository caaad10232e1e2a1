// Declarations shared by the prefill translation units.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace hsd {

// Tiles of the fixed tile order for (T, topk, E, tt): routed, then shared.
int prefill_tile_counts(int T, int topk, int E, int tt, int* nt_routed, int* nt_shared);

// Bytes of one tile's live-K-tile mask: one per 64-column group, rounded up to 8.
__host__ __device__ inline int mask_row_bytes(int kmax) { return (kmax / 64 + 7) / 8 * 8; }

// hc[tile*tt + m, c] = fp16(h[slot's columns][c]) for the rows of non-empty tiles, and
// kmask[tile][mask_row_bytes(kmax)]: 1 iff the tile has a nonzero A value in columns
// [64g, 64g + 64). Routed slot t*topk + k reads row t of h (h_stride elements, default
// topk*F + FS) at column k*F; the shared expert's row of token t is row t of hs (hs_stride
// elements; default: h's columns from topk*F on). Both in h_dtype.
int launch_gather(const void* h, int h_dtype, const int32_t* tile_e, const int32_t* tile_slot, int NT,
                  int tt, int F, int FS, int topk, int E, int kmax, __half* hc, uint8_t* kmask, cudaStream_t st,
                  const void* hs = nullptr, int64_t hs_stride = 0, int64_t h_stride = 0);

// y[t] = sum over the token's first nparts partial rows (+ resid), fixed order.
int launch_reduce(const float* part, const void* resid, void* y, int y_dtype, int T, int D, int topk,
                  int nparts, cudaStream_t st);

// The tensor-core grouped GEMM over the tile order (hsd_prefill_gemm.cu).
// kmask: the gather's live-K-tile bytes; K-tiles whose byte is 0 are skipped. row_dst
// (optional): routed slot s's fp32 output row goes to row_dst[s] instead of part's row;
// shared_out (optional): the shared expert's row of token t goes to shared_out[t * D].
int launch_prefill_gemm(const __half* hc, int kmax, const int32_t* tile_e, const int32_t* tile_slot, int NT,
                        const uint8_t* kmask, const float* gains, const uint32_t* pw, const void* ps, const void* pb, int s_dtype,
                        const uint32_t* spw, const void* sps, const void* spb, float* part, int T, int D,
                        int F, int FS, int topk, int E, cudaStream_t st, float* const* row_dst = nullptr,
                        float* shared_out = nullptr);

// The fixed tile order of build_tiles_kernel: routed tiles over T*topk slots (with nslots_dev,
// only the first *nslots_dev, read on the device), then nt_shared tiles of the shared expert
// over tokens 0 .. T_shared-1.
int launch_build_tiles(const int32_t* sel, int T, int topk, int E, int tt, int nt_routed, int nt_shared,
                       int T_shared, const int* nslots_dev, int32_t* tile_e, int32_t* tile_slot, cudaStream_t st);

constexpr int kPrefillTile = 128;   // slots per tile of the GEMM (its M)

}  // namespace hsd
