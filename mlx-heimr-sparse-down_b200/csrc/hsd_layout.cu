// Load-time layout kernels (hsd/layout.py): the exact nibble transpose of a packed
// 4-bit matrix and the 16-bit transpose of its scales / biases.
//
// nibble_transpose: w [lead, R, CW] u32 (row r, word j packs W[r, 8j .. 8j+7], low nibble
// first) -> out [lead, 8*CW, R/8] (row c, word wo packs W[8wo .. 8wo+7, c]).
// An 8x8 nibble block = 8 input words (rows 8br .. 8br+7 of one word column) = 8
// output words (rows 8j .. 8j+7 of one output word column). A CTA stages a 256-row x
// 32-word input tile in shared memory (coalesced 128-byte row reads, XOR-swizzled
// columns so the block reads are conflict-free), each thread transposes 8x8 nibble
// blocks in registers with three rounds of masked swaps, and writes each output row's
// 32 words (128 bytes) coalesced. HBM-bound: one read and one write of every byte.
#include "hsd_common.cuh"

namespace {

constexpr int kTileR = 256;   // input rows per tile (= 32 output words per output row)
constexpr int kTileW = 32;    // input words per tile row (= 256 output rows)
constexpr int kThreads = 256;

// In-register transpose of an 8x8 matrix of nibbles, a[r] nibble n = M[r][n] ->
// a[n] nibble r = M[r][n]: swap the off-diagonal 4x4, then 2x2, then 1x1 blocks.
__device__ __forceinline__ void transpose8x8_nibbles(uint32_t (&a)[8]) {
#pragma unroll
  for (int r = 0; r < 4; ++r) {   // 4x4 blocks: high 16 bits of rows 0-3 <-> low 16 of rows 4-7
    const uint32_t t = ((a[r] >> 16) ^ a[r + 4]) & 0x0000FFFFu;
    a[r] ^= t << 16;
    a[r + 4] ^= t;
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {   // 2x2 blocks inside each 4x4
    if (r & 2) continue;
    const uint32_t t = ((a[r] >> 8) ^ a[r + 2]) & 0x00FF00FFu;
    a[r] ^= t << 8;
    a[r + 2] ^= t;
  }
#pragma unroll
  for (int r = 0; r < 8; r += 2) {   // single nibbles inside each 2x2
    const uint32_t t = ((a[r] >> 4) ^ a[r + 1]) & 0x0F0F0F0Fu;
    a[r] ^= t << 4;
    a[r + 1] ^= t;
  }
}

__global__ void __launch_bounds__(kThreads) nibble_transpose_kernel(const uint32_t* __restrict__ w,
                                                                    uint32_t* __restrict__ out,
                                                                    int64_t R, int64_t CW) {
  __shared__ uint32_t tile[kTileR * kTileW];   // 32 KB, column index XOR-swizzled by (row / 8)
  const int64_t lead = blockIdx.z;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kTileR;
  const int64_t j0 = static_cast<int64_t>(blockIdx.x) * kTileW;
  const uint32_t* src = w + lead * R * CW;
  uint32_t* dst = out + lead * (CW * 8) * (R / 8);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

  // coalesced tile load: warp reads whole 32-word rows
  for (int rr = warp; rr < kTileR; rr += kThreads / 32) {
    const int64_t r = r0 + rr;
    const int64_t j = j0 + lane;
    uint32_t v = 0;
    if (r < R && j < CW) v = __ldg(src + r * CW + j);
    tile[rr * kTileW + (lane ^ ((rr >> 3) & 31))] = v;
  }
  __syncthreads();

  // each thread: block row br = lane (8 input rows), block columns bw = warp + 8k
  const int br = lane;
  const int64_t orow_words = R / 8;            // words per output row
  const int64_t owc = r0 / 8 + br;             // this block's output word column
#pragma unroll
  for (int k = 0; k < kTileW / (kThreads / 32); ++k) {
    const int bw = warp + k * (kThreads / 32);
    const int64_t j = j0 + bw;
    if (j >= CW) continue;
    if (r0 + 8 * br >= R) continue;            // R % 8 == 0: a block is all in or all out
    uint32_t a[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = 8 * br + i;
      a[i] = tile[rr * kTileW + (bw ^ ((rr >> 3) & 31))];
    }
    transpose8x8_nibbles(a);
#pragma unroll
    for (int n = 0; n < 8; ++n) dst[(8 * j + n) * orow_words + owc] = a[n];
  }
}

// [lead, R, C] 16-bit -> [lead, C, R], 32x32 tiles through padded shared memory.
__global__ void __launch_bounds__(256) swap_last2_u16_kernel(const uint16_t* __restrict__ in,
                                                             uint16_t* __restrict__ out,
                                                             int64_t R, int64_t C) {
  __shared__ uint16_t t[32][33];
  const int64_t lead = blockIdx.z;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  const uint16_t* s = in + lead * R * C;
  uint16_t* d = out + lead * R * C;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int i = ty; i < 32; i += 8) {
    const int64_t r = r0 + i, c = c0 + tx;
    if (r < R && c < C) t[i][tx] = s[r * C + c];
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int64_t c = c0 + i, r = r0 + tx;
    if (r < R && c < C) d[c * R + r] = t[tx][i];
  }
}

}  // namespace

extern "C" int hsd_nibble_transpose(const uint32_t* w, uint32_t* out, int64_t lead, int64_t R,
                                    int64_t CW, void* stream) {
  if (!w || !out) return hsd::set_error(HSD_ERR_ARG, "hsd_nibble_transpose: null pointer");
  if (lead < 1 || R < 8 || CW < 1 || (R % 8) != 0)
    return hsd::set_error(HSD_ERR_SHAPE,
                          "hsd_nibble_transpose: need lead >= 1, R >= 8, R %% 8 == 0, CW >= 1 "
                          "(got lead=%lld R=%lld CW=%lld)",
                          (long long)lead, (long long)R, (long long)CW);
  if (lead > 65535 || (R + kTileR - 1) / kTileR > 65535)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_nibble_transpose: lead or R too large");
  if (w == out) return hsd::set_error(HSD_ERR_ARG, "hsd_nibble_transpose: out aliases w");
  dim3 grid(static_cast<unsigned>((CW + kTileW - 1) / kTileW),
            static_cast<unsigned>((R + kTileR - 1) / kTileR), static_cast<unsigned>(lead));
  nibble_transpose_kernel<<<grid, kThreads, 0, hsd::as_stream(stream)>>>(w, out, R, CW);
  return hsd::check_launch("hsd_nibble_transpose");
}

extern "C" int hsd_swap_last2_u16(const uint16_t* in, uint16_t* out, int64_t lead, int64_t R,
                                  int64_t C, void* stream) {
  if (!in || !out) return hsd::set_error(HSD_ERR_ARG, "hsd_swap_last2_u16: null pointer");
  if (lead < 1 || R < 1 || C < 1 || lead > 65535 || (R + 31) / 32 > 65535)
    return hsd::set_error(HSD_ERR_SHAPE, "hsd_swap_last2_u16: bad shape lead=%lld R=%lld C=%lld",
                          (long long)lead, (long long)R, (long long)C);
  if (in == out) return hsd::set_error(HSD_ERR_ARG, "hsd_swap_last2_u16: out aliases in");
  dim3 grid(static_cast<unsigned>((C + 31) / 32), static_cast<unsigned>((R + 31) / 32),
            static_cast<unsigned>(lead));
  swap_last2_u16_kernel<<<grid, 256, 0, hsd::as_stream(stream)>>>(in, out, R, C);
  return hsd::check_launch("hsd_swap_last2_u16");
}
