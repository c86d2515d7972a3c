/*
 * sage_quant_ref.c — TEST INFRASTRUCTURE ONLY. CPU restatement of the sage_attn pre-pass,
 * used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg as the checker.
 * Nothing in the product links or calls this file.
 *
 * Restates, bit for bit:
 *   - quant_per_block_int8_kernel (kernels/sage_attn/triton_impl.py:7-33), driven the way
 *     per_block_int8 drives it (triton_impl.py:35-82): fp32 input, x *= mult,
 *     scale = max|x| / 127, y = x / scale, y += +-0.5, truncate to int8;
 *   - the optional smoothing k - km of triton_impl.py:39-40 with an fp32 km;
 *   - the K channel mean and V channel absmax statistics of the CUDA pre-pass, in the same
 *     fixed fp64 summation order, so that the GPU's k_mean is reproduced exactly;
 *   - FP8 e4m3 (OCP "E4M3FN": bias 7, no infinities, max 448) round-to-nearest-even with
 *     saturation to +-448, the conversion of the FP8 P.V mode.
 * Built with -ffp-contract=off and without fast-math so every operation is one IEEE
 * binary32/binary64 rounding, like the GPU code.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* One block of `rows` x D values (row-major, fp32) -> int8 + scale. Rows past `valid` are
 * treated as zeros and left untouched in `out` (they are not stored by the reference,
 * triton_impl.py:32). */
static void quant_block(const float* x_in, int valid, int D, float mult, const float* km,
                        int8_t* out, float* scale_out) {
  float amax = 0.0f;
  for (int r = 0; r < valid; ++r)
    for (int d = 0; d < D; ++d) {
      float x = x_in[(size_t)r * D + d];
      if (km) x = x - km[d];
      x = x * mult;
      float a = fabsf(x);
      if (a > amax) amax = a;
    }
  const float scale = amax / 127.0f;
  *scale_out = scale;
  for (int r = 0; r < valid; ++r)
    for (int d = 0; d < D; ++d) {
      float x = x_in[(size_t)r * D + d];
      if (km) x = x - km[d];
      x = x * mult;
      float y = x / scale;
      y = y + ((y >= 0.0f) ? 0.5f : -0.5f);
      int8_t q;
      if (y != y) {
        q = 0; /* 0/0 when the whole block is zero: the conversion yields 0 */
      } else {
        q = (int8_t)(int)truncf(y);
      }
      out[(size_t)r * D + d] = q;
    }
}

/* x: [nheads, S, D] fp32; km: [nheads, D] or NULL; out: [nheads, S, D]; scales: [nheads, ceil(S/blk)] */
void oracle_quant_per_block_int8(const float* x, int64_t nheads, int64_t S, int64_t D, int64_t blk,
                                 float mult, const float* km, int8_t* out, float* scales) {
  const int64_t nb = (S + blk - 1) / blk;
  for (int64_t h = 0; h < nheads; ++h)
    for (int64_t b = 0; b < nb; ++b) {
      const int64_t r0 = b * blk;
      const int valid = (int)((S - r0) < blk ? (S - r0) : blk);
      quant_block(x + (h * S + r0) * D, valid, (int)D, mult, km ? km + h * D : NULL,
                  out + (h * S + r0) * D, scales + h * nb + b);
    }
}

/* Channel mean of K per head in the CUDA pre-pass's summation order:
 * chunk c covers rows [c*chunk, min(S,(c+1)*chunk)); inside a chunk, "thread row" r in
 * [0, rpp) accumulates rows r, r+rpp, ... in increasing order from 0.0; the rpp partials are
 * summed in increasing r from 0.0; chunk sums are summed in increasing c from 0.0;
 * km = (float)(total / S). */
void oracle_k_mean(const float* k, int64_t nheads, int64_t S, int64_t D, int64_t chunk, int64_t rpp,
                   double* scratch /* [rpp*D] */, float* km) {
  for (int64_t h = 0; h < nheads; ++h) {
    const float* kh = k + h * S * D;
    for (int64_t d = 0; d < D; ++d) km[h * D + d] = 0.0f;
    double* total = scratch + rpp * D; /* [D] after the partials */
    for (int64_t d = 0; d < D; ++d) total[d] = 0.0;
    for (int64_t r0 = 0; r0 < S; r0 += chunk) {
      const int64_t r1 = (r0 + chunk < S) ? r0 + chunk : S;
      for (int64_t i = 0; i < rpp * D; ++i) scratch[i] = 0.0;
      for (int64_t r = 0; r < rpp; ++r)
        for (int64_t row = r0 + r; row < r1; row += rpp)
          for (int64_t d = 0; d < D; ++d) scratch[r * D + d] = scratch[r * D + d] + (double)kh[row * D + d];
      for (int64_t d = 0; d < D; ++d) {
        double s = 0.0;
        for (int64_t r = 0; r < rpp; ++r) s = s + scratch[r * D + d];
        total[d] = total[d] + s;
      }
    }
    for (int64_t d = 0; d < D; ++d) km[h * D + d] = (float)(total[d] / (double)S);
  }
}

/* e4m3 encode, round to nearest even, saturating finite values to +-448; NaN -> 0x7F. */
uint8_t oracle_e4m3_encode(float x) {
  if (x != x) return 0x7F;
  const uint8_t sign = signbit(x) ? 0x80 : 0x00;
  float a = fabsf(x);
  if (a == 0.0f) return sign;
  if (a >= 448.0f) return sign | 0x7E;
  if (a < 0.015625f) { /* below 2^-6: subnormal grid of 2^-9 */
    const float q = rintf(a * 512.0f); /* exact scaling, RN-even */
    return sign | (uint8_t)q;         /* q == 8 is the smallest normal, code 0x08 */
  }
  int e;
  float m = frexpf(a, &e); /* a = m * 2^e, m in [0.5, 1) */
  m = m * 2.0f;            /* [1, 2) */
  e = e - 1;
  float f = rintf((m - 1.0f) * 8.0f); /* 0..8 */
  int mi = (int)f;
  if (mi == 8) {
    mi = 0;
    e = e + 1;
  }
  int be = e + 7;
  if (be > 15 || (be == 15 && mi == 7)) return sign | 0x7E;
  return sign | (uint8_t)((be << 3) | mi);
}

float oracle_e4m3_decode(uint8_t c) {
  const float sign = (c & 0x80) ? -1.0f : 1.0f;
  const int be = (c >> 3) & 0xF, mi = c & 7;
  if (be == 15 && mi == 7) return NAN;
  if (be == 0) return sign * ldexpf((float)mi, -9);
  return sign * ldexpf(1.0f + (float)mi / 8.0f, be - 7);
}

/* V [nheads, S, D] fp32 -> per-channel scale = max|v| / 448 and e4m3 codes of v / scale
 * (0 where the channel's scale is 0). */
void oracle_quant_v_fp8(const float* v, int64_t nheads, int64_t S, int64_t D, uint8_t* out, float* scales) {
  for (int64_t h = 0; h < nheads; ++h) {
    const float* vh = v + h * S * D;
    for (int64_t d = 0; d < D; ++d) {
      float m = 0.0f;
      for (int64_t s = 0; s < S; ++s) {
        const float a = fabsf(vh[s * D + d]);
        if (a > m) m = a;
      }
      scales[h * D + d] = m / 448.0f;
    }
    for (int64_t s = 0; s < S; ++s)
      for (int64_t d = 0; d < D; ++d) {
        const float sc = scales[h * D + d];
        const float y = sc > 0.0f ? vh[s * D + d] / sc : 0.0f;
        out[(h * S + s) * D + d] = oracle_e4m3_encode(y);
      }
  }
}
