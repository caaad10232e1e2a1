/*
 * C restatement of the reference's hot path for the CPU (TEST INFRASTRUCTURE ONLY:
 * the checker and the timed CPU baseline; the product never links it).
 *
 * oracle_nibble_transpose  hsd/layout.py:34-50 (unpack, swap, pack), one nibble at a time
 * oracle_sparse_down       the Metal decode kernel's algorithm (hsd/decode.py:37-144):
 *                          per (token, slice of SL neurons): compact the live rows, per
 *                          64-group accumulate acc[o] = sum h*q and hsum = sum h over the
 *                          live rows, out[o] += s*acc + b*hsum (scales / biases read only
 *                          for live groups), part = gain * out; y = sum over slices.
 *                          OpenMP over (token, slice, output block).
 * oracle_dense_down        the dequantised dense path mlx-lm runs (gather_qmm on the
 *                          checkpoint layout: every weight of the selected experts).
 * Scales / biases are bf16 bit patterns.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float bf16f(uint16_t b) {
  union { uint32_t u; float f; } v;
  v.u = ((uint32_t)b) << 16;
  return v.f;
}

/* One nibble at a time; the threads split the output rows (l, c), each of which only its
 * own thread writes. */
void oracle_nibble_transpose(const uint32_t* w, uint32_t* out, int64_t lead, int64_t R, int64_t CW) {
  const int64_t C = CW * 8, OW = R / 8;
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t l = 0; l < lead; ++l)
    for (int64_t c = 0; c < C; ++c) {
      const uint32_t* src = w + l * R * CW;
      uint32_t* dst = out + (l * C + c) * OW;
      memset(dst, 0, sizeof(uint32_t) * (size_t)OW);
      for (int64_t r = 0; r < R; ++r) {
        const uint32_t q = (src[r * CW + c / 8] >> (4 * (c % 8))) & 0xFu;
        dst[r / 8] |= q << (4 * (r % 8));
      }
    }
}

/* One (token, slot, slice) x output words [w_lo, w_hi): adds gain * slice result to yrow. */
static void slice_block(const float* hv, int n, const uint32_t* rows, const uint16_t* sc,
                        const uint16_t* bi, int r0, int D, float gain, int w_lo, int w_hi,
                        float* part, int* live) {
  const int NW = D / 8;
  int nl = 0;
  for (int i = 0; i < n; ++i)
    if (hv[i] != 0.0f) live[nl++] = i;
  for (int o = w_lo * 8; o < w_hi * 8; ++o) part[o] = 0.0f;
  int j = 0;
  while (j < nl) {
    const int g = (r0 + live[j]) / 64;          /* a slice may start inside a 64-group */
    int j1 = j;
    while (j1 < nl && (r0 + live[j1]) / 64 == g) ++j1;
    float hsum = 0.0f;
    for (int t = j; t < j1; ++t) hsum += hv[live[t]];
    const uint16_t* sg = sc + (size_t)g * D;
    const uint16_t* bg = bi + (size_t)g * D;
    for (int w = w_lo; w < w_hi; ++w) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int t = j; t < j1; ++t) {
        const int i = live[t];
        const uint32_t q = rows[(size_t)i * NW + w];
        const float h = hv[i];
        for (int k = 0; k < 8; ++k) acc[k] += h * (float)((q >> (4 * k)) & 0xFu);
      }
      for (int k = 0; k < 8; ++k) part[w * 8 + k] += bf16f(sg[w * 8 + k]) * acc[k] + bf16f(bg[w * 8 + k]) * hsum;
    }
    j = j1;
  }
  for (int o = w_lo * 8; o < w_hi * 8; ++o) part[o] *= gain;
}

/* h [B, topk*F+FS] f32, sel [B, topk], gains [B, topk+1]; pw [E, F, D/8], ps / pb
 * [E, F/64, D] bf16 bits; spw [FS, D/8], sps / spb [FS/64, D] -> y [B, D] f32.
 * SL: neurons per slice (divides F and FS). nthreads <= 0: OpenMP default. */
void oracle_sparse_down(const float* h, const int32_t* sel, const float* gains, const uint32_t* pw,
                        const uint16_t* ps, const uint16_t* pb, const uint32_t* spw,
                        const uint16_t* sps, const uint16_t* spb, float* y, int B, int D, int F,
                        int FS, int topk, int SL, int nthreads) {
  const int NW = D / 8, NR = topk * F + FS;
  const int SPE = F / SL, NSS = FS / SL, NS = topk * SPE + NSS;
  const int NBLK = 4;                                  /* output blocks per slice */
  float* part = (float*)calloc((size_t)B * NS * D, sizeof(float));
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
#pragma omp parallel
  {
    int* live = (int*)malloc(sizeof(int) * (size_t)(F > FS ? F : FS));
#pragma omp for schedule(dynamic, 1) collapse(3)
    for (int b = 0; b < B; ++b)
      for (int s = 0; s < NS; ++s)
        for (int blk = 0; blk < NBLK; ++blk) {
          const int w_lo = (int)((int64_t)NW * blk / NBLK), w_hi = (int)((int64_t)NW * (blk + 1) / NBLK);
          float* pp = part + ((size_t)b * NS + s) * D;
          if (s < topk * SPE) {
            const int k = s / SPE, r0 = (s % SPE) * SL;
            const int e = sel[b * topk + k];
            slice_block(h + (size_t)b * NR + (size_t)k * F + r0, SL, pw + ((size_t)e * F + r0) * NW,
                        ps + (size_t)e * (F / 64) * D, pb + (size_t)e * (F / 64) * D, r0, D,
                        gains[b * (topk + 1) + k], w_lo, w_hi, pp, live);
          } else {
            const int r0 = (s - topk * SPE) * SL;
            slice_block(h + (size_t)b * NR + (size_t)topk * F + r0, SL, spw + (size_t)r0 * NW, sps, spb,
                        r0, D, gains[b * (topk + 1) + topk], w_lo, w_hi, pp, live);
          }
        }
    free(live);
  }
  for (int b = 0; b < B; ++b)
    for (int o = 0; o < D; ++o) {
      float t = 0.0f;
      for (int s = 0; s < NS; ++s) t += part[((size_t)b * NS + s) * D + o];
      y[(size_t)b * D + o] = t;
    }
  free(part);
}

/* The dense dequantised path on the checkpoint layout: w [E, D, F/8], s / b [E, D, F/64];
 * sw [D, FS/8], ss / sb [D, FS/64] -> y [B, D] f32. */
void oracle_dense_down(const float* h, const int32_t* sel, const float* gains, const uint32_t* w,
                       const uint16_t* s, const uint16_t* bb, const uint32_t* sw, const uint16_t* ss,
                       const uint16_t* sb, float* y, int B, int D, int F, int FS, int topk, int nthreads) {
  const int NR = topk * F + FS;
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#endif
#pragma omp parallel for schedule(static) collapse(2)
  for (int b = 0; b < B; ++b)
    for (int o = 0; o < D; ++o) {
      float tot = 0.0f;
      for (int k = 0; k <= topk; ++k) {
        const int width = (k < topk) ? F : FS;
        const uint32_t* wr = (k < topk) ? w + ((size_t)sel[b * topk + k] * D + o) * (F / 8) : sw + (size_t)o * (FS / 8);
        const uint16_t* sr = (k < topk) ? s + ((size_t)sel[b * topk + k] * D + o) * (F / 64) : ss + (size_t)o * (FS / 64);
        const uint16_t* br = (k < topk) ? bb + ((size_t)sel[b * topk + k] * D + o) * (F / 64) : sb + (size_t)o * (FS / 64);
        const float* hv = h + (size_t)b * NR + (size_t)k * F;
        float acc = 0.0f;
        for (int g = 0; g < width / 64; ++g) {
          const float sc = bf16f(sr[g]), bi = bf16f(br[g]);
          for (int j = 0; j < 64; ++j) {
            const int i = g * 64 + j;
            const float q = (float)((wr[i / 8] >> (4 * (i % 8))) & 0xFu);
            acc += (sc * q + bi) * hv[i];
          }
        }
        tot += gains[b * (topk + 1) + k] * acc;
      }
      y[(size_t)b * D + o] = tot;
    }
}
