/*
 * CPU oracle for the packed weight formats. TEST INFRASTRUCTURE ONLY: the tests, the smoke check
 * and the CPU-baseline leg of the benchmark link this file; the product never does.
 *
 * A plain-C restatement of the reference's format code, written to be read against it:
 *   pack_int4     kernels/quant.py:20-28   8 values along K -> one int32, value i in bits 4i..4i+3
 *   unpack_int4   kernels/quant.py:31-35   (p >> 4i) & 0xF
 *   quantize_rtn  kernels/quant.py:38-49   per (group of G along K, column): fp32 min/max,
 *                                          scale = (max-min)/15 clamped >= 1e-6,
 *                                          zero = round(-min/scale) clamped to [0,15],
 *                                          q = round(w/scale + zero) clamped to [0,15],
 *                                          round = half-to-even, scale/zero stored as fp16
 *   quantize_fp8  kernels/fp8.py:25-30     per output row: scale = absmax/448 clamped >= 1e-12,
 *                                          wq = e4m3fn(clamp(w/scale, +-448)), stored [K, N]
 *   dequantize_fp8 kernels/fp8.py:33-35    fp16(fp32(wq) * fp32(scale))
 *
 * All fp32 arithmetic is IEEE (the build passes -ffp-contract=off, no fast-math), which is what
 * the reference's torch CPU ops do. fp16 conversion uses the C `_Float16` type (round to nearest
 * even). The e4m3fn encoder below is written from the format's definition (1 sign bit, 4
 * exponent bits with bias 7, 3 mantissa bits, no infinities, 0x7F = NaN, max finite 448).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float h2f(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static uint16_t f2h(float f) {
  _Float16 v = (_Float16)f;
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

/* torch.clamp(x, lo, hi) == min(max(x, lo), hi) with the comparison order of at::clamp. */
static float clampf(float x, float lo, float hi) {
  float y = (x < lo) ? lo : x;
  return (y > hi) ? hi : y;
}

void oracle_pack_int4(const int32_t* q, int64_t K, int64_t N, int32_t* packed) {
  for (int64_t r = 0; r < K / 8; ++r)
    for (int64_t n = 0; n < N; ++n) {
      uint64_t acc = 0;
      for (int i = 0; i < 8; ++i) acc += (uint64_t)(int64_t)q[(r * 8 + i) * N + n] << (4 * i);
      packed[r * N + n] = (int32_t)(uint32_t)acc;
    }
}

void oracle_unpack_int4(const int32_t* packed, int64_t K, int64_t N, int32_t* q) {
  for (int64_t r = 0; r < K / 8; ++r)
    for (int64_t n = 0; n < N; ++n)
      for (int i = 0; i < 8; ++i) q[(r * 8 + i) * N + n] = (packed[r * N + n] >> (4 * i)) & 0xF;
}

/* w: fp16 [N, K] row-major. qweight: int32 [K/8, N]; scales, zeros: fp16 [K/G, N]. */
void oracle_quantize_rtn(const uint16_t* w, int64_t N, int64_t K, int64_t G, int32_t* qweight,
                         uint16_t* scales, uint16_t* zeros) {
  for (int64_t g = 0; g < K / G; ++g)
    for (int64_t n = 0; n < N; ++n) {
      const uint16_t* row = w + n * K + g * G;
      float mn = h2f(row[0]), mx = mn;
      for (int64_t k = 1; k < G; ++k) {
        float v = h2f(row[k]);
        mn = v < mn ? v : mn;
        mx = v > mx ? v : mx;
      }
      float scale = (mx - mn) / 15.0f;
      scale = scale < 1e-6f ? 1e-6f : scale;
      float zero = clampf(nearbyintf(-mn / scale), 0.0f, 15.0f);
      for (int64_t k = 0; k < G; k += 8) {
        uint32_t word = 0;
        for (int i = 0; i < 8; ++i) {
          float q = clampf(nearbyintf(h2f(row[k + i]) / scale + zero), 0.0f, 15.0f);
          word |= (uint32_t)(int32_t)q << (4 * i);
        }
        qweight[((g * G + k) / 8) * N + n] = (int32_t)word;
      }
      scales[g * N + n] = f2h(scale);
      zeros[g * N + n] = f2h(zero);
    }
}

/* fp16 dequantization of the packed format, [N, K] like nn.Linear.weight (reference.py:27-36):
 * (fp16(q) - z) * s with fp16 rounding after each op. */
void oracle_dequantize_int4(const int32_t* qweight, const uint16_t* scales, const uint16_t* zeros,
                            int64_t N, int64_t K, int64_t G, uint16_t* w) {
  for (int64_t k = 0; k < K; ++k)
    for (int64_t n = 0; n < N; ++n) {
      int32_t q = (qweight[(k / 8) * N + n] >> (4 * (k % 8))) & 0xF;
      _Float16 s, z;
      memcpy(&s, &scales[(k / G) * N + n], 2);
      memcpy(&z, &zeros[(k / G) * N + n], 2);
      _Float16 d = (_Float16)((float)q - (float)z); /* exact: small integers */
      _Float16 v = (_Float16)((float)d * (float)s); /* one rounding of the exact product */
      memcpy(&w[n * K + k], &v, 2);
    }
}

/* float -> e4m3fn, round to nearest even; |f| must already be <= 448 (the reference clamps). */
uint8_t oracle_f32_to_e4m3(float f) {
  uint8_t sign = signbit(f) ? 0x80 : 0x00;
  float a = fabsf(f);
  if (isnan(f)) return 0x7F;
  if (a == 0.0f) return sign;
  int e;
  frexpf(a, &e);              /* a = m * 2^e, m in [0.5, 1): floor(log2 a) = e - 1 */
  int E = e - 1;
  if (E < -6) E = -6;         /* subnormals share the quantum of the smallest normal binade */
  float quantum = ldexpf(1.0f, E - 3);
  float n = nearbyintf(a / quantum); /* exact scaling by a power of two, then RNE */
  float v = n * quantum;
  if (v > 448.0f) return sign | 0x7F; /* not reachable after the reference's clamp */
  if (v < ldexpf(1.0f, -6)) return sign | (uint8_t)(v / ldexpf(1.0f, -9)); /* subnormal */
  frexpf(v, &e);
  E = e - 1;
  int m = (int)(v / ldexpf(1.0f, E - 3)) - 8;
  return sign | (uint8_t)(((E + 7) << 3) | m);
}

float oracle_e4m3_to_f32(uint8_t b) {
  int e = (b >> 3) & 0xF, m = b & 7;
  float v;
  if ((b & 0x7F) == 0x7F) return NAN;
  if (e == 0) v = ldexpf((float)m, -9);
  else v = ldexpf((float)(8 + m), e - 10);
  return (b & 0x80) ? -v : v;
}

/* w: fp16 [N, K]. wq: e4m3 bytes [K, N]; scale: fp16 [N]. */
void oracle_quantize_fp8(const uint16_t* w, int64_t N, int64_t K, uint8_t* wq, uint16_t* scale) {
  for (int64_t n = 0; n < N; ++n) {
    float amax = 0.0f;
    for (int64_t k = 0; k < K; ++k) {
      float v = fabsf(h2f(w[n * K + k]));
      amax = v > amax ? v : amax;
    }
    float s = amax / 448.0f;
    s = s < 1e-12f ? 1e-12f : s;
    for (int64_t k = 0; k < K; ++k)
      wq[k * N + n] = oracle_f32_to_e4m3(clampf(h2f(w[n * K + k]) / s, -448.0f, 448.0f));
    scale[n] = f2h(s);
  }
}

/* wq: e4m3 [K, N], scale fp16 [N] -> fp16 [N, K]. */
void oracle_dequantize_fp8(const uint8_t* wq, const uint16_t* scale, int64_t N, int64_t K,
                           uint16_t* w) {
  for (int64_t n = 0; n < N; ++n)
    for (int64_t k = 0; k < K; ++k)
      w[n * K + k] = f2h(oracle_e4m3_to_f32(wq[k * N + n]) * h2f(scale[n]));
}
