// Decode attention of a GQA layer over a fixed-size cache with a device-side position: the
// decode-row form of the reference model's attention block (mlx-lm nemotron_h, no positional
// encoding), for decode steps replayed from a captured graph whose shapes cannot follow the
// context length.
//
//   q   [L, QH*HD] (row stride q_stride)       row l = the token at position pos + l
//   kc  [KVH, max_len, HD], vc the same          the cache, rows pos .. pos+L-1 already written
//   out [L, QH*HD]                               out[l, h] = softmax(q_h . K[0..n) / sqrt(HD)) V
//   with n = pos + l + 1 keys for row l (causal), query head h reading KV head h / (QH/KVH).
//
// Split over the keys in chunks of 64 (flash-decoding): one block per (chunk, KV head, row)
// loads the chunk's K and V rows once into shared memory with 16-byte loads and serves all
// G = QH/KVH query heads of the KV head from there -- scores, the chunk's max and exp-sum,
// and the unnormalised output -- into an fp32 workspace; a second kernel merges the chunks
// of each (row, head) in chunk order. A row's result depends only on its query and its n,
// never on the other rows of the launch, so a verify row equals the same token alone.
#include "hsd_common.cuh"

HSD_DEFINE_STATUS(attn)

namespace {

constexpr int kChunk = 64;        // keys per block
constexpr int kThreads = 256;
constexpr int kMaxG = 16;         // query heads per KV head
constexpr int kMaxHD = 128;       // head dim: 128 (the reference model's) or 64
constexpr int kRec = 4;           // floats after a chunk's output: max, exp-sum, 2 pad (16-byte records)

__device__ __forceinline__ void bf16x8_to_f32(const uint4 r, float* v) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = __uint_as_float(w[k] << 16);
    v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}

__device__ __forceinline__ int keys_of_row(const int64_t* pos, int l, int max_len) {
  const int64_t n = *pos + l + 1;
  if (n > max_len) {
    if (threadIdx.x == 0) atomicCAS(&hsd_status_word_attn, 0, HSD_ERR_INDEX);
    return max_len;
  }
  return static_cast<int>(n);
}

// ws layout: [L, QH, nsplit, kHD + kRec] fp32: the chunk's unnormalised output, its max, its
// exp-sum (records of a multiple of 16 bytes, so every record's float4 stores are aligned)
template <int kHD>
__global__ void __launch_bounds__(kThreads) attn_chunk_kernel(const __nv_bfloat16* __restrict__ q, int64_t q_stride,
                                                              const __nv_bfloat16* __restrict__ kc,
                                                              const __nv_bfloat16* __restrict__ vc,
                                                              const int64_t* pos, int QH, int KVH, int max_len,
                                                              int nsplit, float scale, float* ws) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  constexpr int kRowPad = kHD + 8;  // bf16 per staged K / V row (16-byte skew between rows)
  __shared__ __align__(16) __nv_bfloat16 ks[kChunk * kRowPad];
  __shared__ __align__(16) __nv_bfloat16 vs[kChunk * kRowPad];
  __shared__ __align__(16) float qs[kMaxG * kHD];
  __shared__ float ps[kMaxG * kChunk];
  const int split = blockIdx.x, kvh = blockIdx.y, l = blockIdx.z;
  const int tid = threadIdx.x;
  const int G = QH / KVH;
  const int n = keys_of_row(pos, l, max_len);
  const int j0 = split * kChunk;
  if (j0 >= n) return;
  const int nk = min(kChunk, n - j0);

  // the chunk's K / V rows and the G query rows, 16 bytes per load
  const int64_t cbase = (static_cast<int64_t>(kvh) * max_len + j0) * kHD;
  for (int t = tid; t < nk * (kHD / 8); t += kThreads) {
    const int j = t / (kHD / 8), c = t % (kHD / 8);
    *reinterpret_cast<uint4*>(&ks[j * kRowPad + c * 8]) = __ldg(reinterpret_cast<const uint4*>(kc + cbase + j * kHD) + c);
    *reinterpret_cast<uint4*>(&vs[j * kRowPad + c * 8]) = __ldg(reinterpret_cast<const uint4*>(vc + cbase + j * kHD) + c);
  }
  for (int t = tid; t < G * (kHD / 8); t += kThreads) {
    const int h = t / (kHD / 8), c = t % (kHD / 8);
    float v[8];
    bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(q + l * q_stride + static_cast<int64_t>(kvh * G + h) * kHD) + c), v);
#pragma unroll
    for (int i = 0; i < 8; ++i) qs[h * kHD + c * 8 + i] = v[i];
  }
  __syncthreads();

  // scores: thread (h = tid / 16, jj = tid % 16) takes keys jj, jj+16, jj+32, jj+48
  const int h = tid >> 4, jj = tid & 15;
  float s[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) s[k] = -INFINITY;
  if (h < G) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = jj + 16 * k;
      if (j < nk) {
        float acc = 0.f;
#pragma unroll 4
        for (int c = 0; c < kHD / 8; ++c) {
          float kv[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(&ks[j * kRowPad + c * 8]), kv);
          const float4 qa = *reinterpret_cast<const float4*>(&qs[h * kHD + c * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&qs[h * kHD + c * 8 + 4]);
          acc = fmaf(qa.x, kv[0], acc); acc = fmaf(qa.y, kv[1], acc);
          acc = fmaf(qa.z, kv[2], acc); acc = fmaf(qa.w, kv[3], acc);
          acc = fmaf(qb.x, kv[4], acc); acc = fmaf(qb.y, kv[5], acc);
          acc = fmaf(qb.z, kv[6], acc); acc = fmaf(qb.w, kv[7], acc);
        }
        s[k] = acc * scale;
      }
    }
  }
  // the chunk's max and exp-sum per head over its 16 lanes (a half warp)
  float m = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float e = (s[k] == -INFINITY) ? 0.f : expf(s[k] - m);
    if (h < G) ps[h * kChunk + jj + 16 * k] = e;
    sum += e;
  }
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __syncthreads();

  // unnormalised output: thread (h, 8 dims d0 = jj*8) sums p_hj * v_j over the chunk
  if (h < G && jj * 8 < kHD) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    const int d0 = jj * 8;
    for (int j = 0; j < nk; ++j) {
      const float p = ps[h * kChunk + j];
      float vv[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(&vs[j * kRowPad + d0]), vv);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(p, vv[i], acc[i]);
    }
    float* dst = ws + ((static_cast<int64_t>(l) * QH + kvh * G + h) * nsplit + split) * (kHD + kRec);
    *reinterpret_cast<float4*>(dst + d0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(dst + d0 + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    if (jj == 0) {
      dst[kHD] = m;
      dst[kHD + 1] = sum;
    }
  }
}

// out[l, h, d] = sum_s o_s[d] e^{m_s - M} / sum_s l_s e^{m_s - M}, chunks in order
template <int kHD>
__global__ void __launch_bounds__(kHD) attn_merge_kernel(const float* __restrict__ ws, const int64_t* pos, int QH,
                                                        int max_len, int nsplit, __nv_bfloat16* out) {
  hsd::pdl_launch_dependents();   // the next kernel may launch now
  hsd::pdl_wait();                // inputs of earlier kernels are visible from here
  const int h = blockIdx.x, l = blockIdx.y, d = threadIdx.x;
  const int n = keys_of_row(pos, l, max_len);
  const int ns = (n + kChunk - 1) / kChunk;
  const float* base = ws + (static_cast<int64_t>(l) * QH + h) * nsplit * (kHD + kRec);
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, base[s * (kHD + kRec) + kHD]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < ns; ++s) {
    const float w = expf(base[s * (kHD + kRec) + kHD] - M);
    num = fmaf(base[s * (kHD + kRec) + d], w, num);
    den = fmaf(base[s * (kHD + kRec) + kHD + 1], w, den);
  }
  out[(static_cast<int64_t>(l) * QH + h) * kHD + d] = __float2bfloat16_rn(num / den);
}

}  // namespace

extern "C" int hsd_attn_decode_workspace_bytes(int L, int QH, int max_len, size_t* bytes) {
  if (!bytes || L < 1 || QH < 1 || max_len < 1) return hsd::set_error(HSD_ERR_ARG, "hsd_attn_decode_workspace_bytes: bad argument");
  const size_t nsplit = (static_cast<size_t>(max_len) + kChunk - 1) / kChunk;
  *bytes = static_cast<size_t>(L) * QH * nsplit * (kMaxHD + kRec) * sizeof(float);
  return HSD_OK;
}

extern "C" int hsd_attn_decode(const void* q, int64_t q_stride, const void* kc, const void* vc, const int64_t* pos,
                               void* out, float* ws, int L, int QH, int KVH, int HD, int max_len, float scale,
                               void* stream) {
  const char* who = "hsd_attn_decode";
  if (!q || !kc || !vc || !pos || !out || !ws) return hsd::set_error(HSD_ERR_ARG, "%s: null pointer", who);
  if ((HD != 128 && HD != 64) || L < 1 || L > 65535 || KVH < 1 || QH % KVH != 0 || QH / KVH > kMaxG ||
      max_len < 1 || q_stride < static_cast<int64_t>(QH) * HD || q_stride % 8 != 0)
    return hsd::set_error(HSD_ERR_SHAPE, "%s: need HD 64 or 128, QH %% KVH == 0, QH/KVH <= %d, q_stride %% 8 == 0",
                          who, kMaxG);
  if (!hsd::aligned(q, 16) || !hsd::aligned(kc, 16) || !hsd::aligned(vc, 16) || !hsd::aligned(ws, 16))
    return hsd::set_error(HSD_ERR_ALIGN, "%s: q, caches and workspace must be 16-byte aligned", who);
  const int nsplit = (max_len + kChunk - 1) / kChunk;
  cudaStream_t st = hsd::as_stream(stream);
  const auto* qb = static_cast<const __nv_bfloat16*>(q);
  const auto* kb = static_cast<const __nv_bfloat16*>(kc);
  const auto* vb = static_cast<const __nv_bfloat16*>(vc);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  if (HD == 128) {
    hsd::launch_pdl(attn_chunk_kernel<128>, dim3(nsplit, KVH, L), dim3(kThreads), 0, st, qb, q_stride, kb, vb, pos, QH, KVH, max_len,
                                                                        nsplit, scale, ws);
    int rc = hsd::check_launch(who);
    if (rc != HSD_OK) return rc;
    hsd::launch_pdl(attn_merge_kernel<128>, dim3(QH, L), dim3(128), 0, st, ws, pos, QH, max_len, nsplit, ob);
  } else {
    hsd::launch_pdl(attn_chunk_kernel<64>, dim3(nsplit, KVH, L), dim3(kThreads), 0, st, qb, q_stride, kb, vb, pos, QH, KVH, max_len,
                                                                       nsplit, scale, ws);
    int rc = hsd::check_launch(who);
    if (rc != HSD_OK) return rc;
    hsd::launch_pdl(attn_merge_kernel<64>, dim3(QH, L), dim3(64), 0, st, ws, pos, QH, max_len, nsplit, ob);
  }
  return hsd::check_launch(who);
}
