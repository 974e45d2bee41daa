/*
 * ts_oracle_kernels.c — CPU restatement of the WASM kernels.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker + timed CPU baseline); never part
 * of the shipped CUDA backend.  Line citations are into
 * packages/textsift/src/zig/wasm_exports.zig unless stated otherwise.
 *
 * Conventions that make this bit-exact against the reference:
 *   - "fma4" (c/fma.c:10-13, relaxed_madd) is a fused multiply-add: fmaf().
 *   - Every other a*b+c is a rounded multiply followed by a rounded add; the
 *     Makefile passes -ffp-contract=off so gcc never fuses them.
 *   - 4-lane SIMD loops are written as explicit lane arrays so that each lane
 *     accumulates in exactly the reference's order, and horizontal sums use
 *     the reference's association.
 *   - @exp is the C library expf (Zig lowers @exp on f32 to a correctly
 *     rounded-in-practice expf; differences are at most 1 ulp and only reach
 *     the attention tail entries and the router softmax).
 */
#include "ts_oracle.h"

#include <immintrin.h>
#include <math.h>
#include <string.h>

static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* math.zig:45-52 */
float tso_f16_to_f32(uint16_t bits) {
  uint32_t u = bits;
  uint32_t sign_shifted = (u & 0x8000u) << 16;
  uint32_t rest = u & 0x7fffu;
  uint32_t biased = rest == 0 ? 0u : (rest << 13) + (112u << 23);
  return bits_f32(sign_shifted | biased);
}

/* math.zig:54-82 */
uint16_t tso_f32_to_f16(float f) {
  uint32_t u = f32_bits(f);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t exp32 = (u >> 23) & 0xffu;
  uint32_t mant = u & 0x7fffffu;
  if (exp32 == 0xffu) return (uint16_t)(sign | 0x7c00u | (mant != 0 ? 0x200u : 0u));
  int32_t e16 = (int32_t)exp32 - 127 + 15;
  if (e16 >= 0x1f) return (uint16_t)(sign | 0x7c00u);
  if (e16 <= 0) {
    if (e16 < -10) return (uint16_t)sign;
    uint32_t shift = (uint32_t)(14 - e16);
    uint32_t mant24 = mant | 0x800000u;
    uint32_t rounded = (mant24 + (1u << (shift - 1))) >> shift;
    return (uint16_t)(sign | rounded);
  }
  uint32_t lsb = (mant >> 13) & 1u;
  uint32_t m10 = (mant + 0xfffu + lsb) >> 13;
  uint32_t ue = (uint32_t)e16;
  if (m10 >= 0x400u) {
    m10 = 0;
    ue += 1;
    if (ue >= 0x1fu) return (uint16_t)(sign | 0x7c00u);
  }
  return (uint16_t)(sign | (ue << 10) | m10);
}

/* math.zig:13-16 */
float tso_bf16_to_f32(uint16_t b) { return bits_f32((uint32_t)b << 16); }

/* math.zig:19-28 */
uint16_t tso_f32_to_bf16(float f) {
  uint32_t bits = f32_bits(f);
  if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu) != 0)
    return (uint16_t)((bits | 0x00400000u) >> 16);
  uint32_t rounded = bits + 0x7FFFu + ((bits >> 16) & 1u);
  return (uint16_t)(rounded >> 16);
}

/* browser/backends/wasm.ts:264-291 and browser/inference/rope.ts:78-104:
 * the JS variant rounds the double to f32 first and maps ±0 to +0. */
uint16_t tso_js_f32_to_f16(double d) {
  if (d == 0.0) return 0;
  return tso_f32_to_f16((float)d);
}

/* browser/backends/wasm.ts:776-797: exact fp16 -> f32 widen of the logits. */
float tso_js_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  if (e == 0) {
    if (mant == 0) return bits_f32(sign);
    int ee = 1;
    uint32_t m = mant;
    while ((m & 0x400u) == 0) { m <<= 1; ee--; }
    m &= 0x3ffu;
    return bits_f32(sign | ((uint32_t)(ee + 112) << 23) | (m << 13));
  }
  if (e == 0x1f) return bits_f32(sign | 0x7f800000u | (mant << 13));
  return bits_f32(sign | ((e + 112u) << 23) | (mant << 13));
}

/* ------------------------------------------------------------------ */
/* RMSNorm family                                                      */
/* ------------------------------------------------------------------ */

/* wasm_exports.zig:186-218 (scalar; only used by the fixture test) */
void tso_rms_norm(const uint16_t* x, const uint16_t* gamma, uint16_t* out,
                  uint32_t T, uint32_t D, float eps) {
  const float d_inv = 1.0f / (float)D;
  for (uint32_t t = 0; t < T; t++) {
    const uint16_t* row = x + (size_t)t * D;
    float sumsq = 0.0f;
    for (uint32_t d = 0; d < D; d++) {
      float v = tso_f16_to_f32(row[d]);
      float sq = v * v;
      sumsq = sumsq + sq;
    }
    float inv_rms = 1.0f / sqrtf(sumsq * d_inv + eps);
    for (uint32_t d = 0; d < D; d++) {
      float xv = tso_f16_to_f32(row[d]);
      float gv = tso_f16_to_f32(gamma[d]);
      float a = xv * inv_rms;
      out[(size_t)t * D + d] = tso_f32_to_f16(a * gv);
    }
  }
}

/* wasm_exports.zig:229-277: 4-lane partial sums of squares, then a scalar tail. */
void tso_rms_norm_fp16_to_f32(const uint16_t* x, const uint16_t* gamma, float* out,
                              uint32_t T, uint32_t D, float eps) {
  const float d_inv = 1.0f / (float)D;
  for (uint32_t t = 0; t < T; t++) {
    const uint16_t* row = x + (size_t)t * D;
    float* orow = out + (size_t)t * D;
    float s[4] = {0, 0, 0, 0};
    uint32_t d = 0;
    for (; d + 4 <= D; d += 4)
      for (int l = 0; l < 4; l++) {
        float v = tso_f16_to_f32(row[d + l]);
        float sq = v * v;
        s[l] = s[l] + sq;
      }
    float sumsq = s[0] + s[1] + s[2] + s[3];
    for (; d < D; d++) {
      float v = tso_f16_to_f32(row[d]);
      float sq = v * v;
      sumsq = sumsq + sq;
    }
    float inv_rms = 1.0f / sqrtf(sumsq * d_inv + eps);
    for (d = 0; d < D; d++) {
      float a = tso_f16_to_f32(row[d]) * inv_rms;
      orow[d] = a * tso_f16_to_f32(gamma[d]);
    }
  }
}

/* wasm_exports.zig:288-350: sum of squares uses the UNROUNDED f32 sum; the
 * normalised output re-reads the fp16-rounded sum. */
void tso_add_rmsnorm_fp16_to_f32(const uint16_t* a, const uint16_t* b, const uint16_t* gamma,
                                 uint16_t* sum_out, float* norm_out,
                                 uint32_t T, uint32_t D, float eps) {
  const float d_inv = 1.0f / (float)D;
  for (uint32_t t = 0; t < T; t++) {
    const uint16_t* ar = a + (size_t)t * D;
    const uint16_t* br = b + (size_t)t * D;
    uint16_t* sr = sum_out + (size_t)t * D;
    float* nr = norm_out + (size_t)t * D;
    float s[4] = {0, 0, 0, 0};
    uint32_t d = 0;
    for (; d + 4 <= D; d += 4)
      for (int l = 0; l < 4; l++) {
        float sv = tso_f16_to_f32(ar[d + l]) + tso_f16_to_f32(br[d + l]);
        sr[d + l] = tso_f32_to_f16(sv);
        float sq = sv * sv;
        s[l] = s[l] + sq;
      }
    float sumsq = s[0] + s[1] + s[2] + s[3];
    for (; d < D; d++) {
      float sv = tso_f16_to_f32(ar[d]) + tso_f16_to_f32(br[d]);
      sr[d] = tso_f32_to_f16(sv);
      float sq = sv * sv;
      sumsq = sumsq + sq;
    }
    float inv_rms = 1.0f / sqrtf(sumsq * d_inv + eps);
    for (d = 0; d < D; d++) {
      float x = tso_f16_to_f32(sr[d]) * inv_rms;
      nr[d] = x * tso_f16_to_f32(gamma[d]);
    }
  }
}

/* ------------------------------------------------------------------ */
/* Top-k / softmax                                                     */
/* ------------------------------------------------------------------ */

/* wasm_exports.zig:367-426: seed with the first k, insertion-sort
 * descending with strict '>', then replace-last-and-bubble. */
void tso_topk_partial_f32(const float* x, int32_t* out_idx, float* out_val,
                          uint32_t rows, uint32_t cols, uint32_t k) {
  for (uint32_t r = 0; r < rows; r++) {
    const float* row = x + (size_t)r * cols;
    int32_t* oi = out_idx + (size_t)r * k;
    float* ov = out_val + (size_t)r * k;
    for (uint32_t i = 0; i < k; i++) { oi[i] = (int32_t)i; ov[i] = row[i]; }
    for (uint32_t s = 1; s < k; s++) {
      uint32_t j = s;
      while (j > 0 && ov[j] > ov[j - 1]) {
        float tv = ov[j]; ov[j] = ov[j - 1]; ov[j - 1] = tv;
        int32_t ti = oi[j]; oi[j] = oi[j - 1]; oi[j - 1] = ti;
        j--;
      }
    }
    for (uint32_t c = k; c < cols; c++) {
      float v = row[c];
      if (v > ov[k - 1]) {
        ov[k - 1] = v;
        oi[k - 1] = (int32_t)c;
        uint32_t j = k - 1;
        while (j > 0 && ov[j] > ov[j - 1]) {
          float tv = ov[j]; ov[j] = ov[j - 1]; ov[j - 1] = tv;
          int32_t ti = oi[j]; oi[j] = oi[j - 1]; oi[j - 1] = ti;
          j--;
        }
      }
    }
  }
}

/* wasm_exports.zig:919-958 */
void tso_softmax_f32(const float* x, float* out, uint32_t rows, uint32_t cols) {
  for (uint32_t r = 0; r < rows; r++) {
    const float* row = x + (size_t)r * cols;
    float* o = out + (size_t)r * cols;
    float m = row[0];
    for (uint32_t c = 1; c < cols; c++) if (row[c] > m) m = row[c];
    float sum = 0.0f;
    for (uint32_t c = 0; c < cols; c++) {
      float e = expf(row[c] - m);
      o[c] = e;
      sum = sum + e;
    }
    float inv = sum > 0.0f ? 1.0f / sum : 1.0f / (float)cols;
    for (uint32_t c = 0; c < cols; c++) o[c] = o[c] * inv;
  }
}

/* ------------------------------------------------------------------ */
/* MatMulNBits (int4 block-32)                                          */
/* ------------------------------------------------------------------ */

/* wasm_exports.zig:512-540: element k of a 32-block is byte k/2, low nibble
 * for even k.  wasm_exports.zig:545-548: even blocks' zp in the low nibble. */
static inline void decode_block(const uint8_t* w_row, uint32_t block_d, uint8_t zp, float q[32]) {
  const uint8_t* p = w_row + block_d / 2;
  for (int i = 0; i < 16; i++) {
    q[2 * i] = (float)((int)(p[i] & 0x0F) - (int)zp);
    q[2 * i + 1] = (float)((int)((p[i] >> 4) & 0x0F) - (int)zp);
  }
}
static inline uint8_t extract_zp(const uint8_t* zp_row, uint32_t b) {
  uint8_t byte = zp_row[b >> 1];
  return (b & 1) == 0 ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
}

static inline float load_x(int x_is_f32, const void* x, size_t i) {
  return x_is_f32 ? ((const float*)x)[i] : tso_f16_to_f32(((const uint16_t*)x)[i]);
}
static inline void store_out(int out_is_f32, void* out, size_t i, float v) {
  if (out_is_f32) ((float*)out)[i] = v;
  else ((uint16_t*)out)[i] = tso_f32_to_f16(v);
}

/* wasm_exports.zig:560-708.  Rows below 8*floor(T/8) take the 8-row tile
 * path (615-652): lane l accumulates fma(x[4c+l], q[4c+l]) for c = 0..7,
 * block sum (v0+v1)+(v2+v3), then sum += bsum*scale (mul, then add).
 * Remaining rows take the tail path (669-707): a0 takes the even 4-chunks,
 * a1 the odd ones, c = a0+a1, acc += ((c0+c1)+(c2+c3))*scale. */
void tso_matmul_int4_scalar(int x_is_f32, int out_is_f32, const void* x,
                            const uint8_t* w_int4, const uint16_t* w_scales, const uint8_t* w_zp,
                            const uint16_t* bias, void* out, uint32_t T, uint32_t N, uint32_t D) {
  const uint32_t BLOCK = 32, TR = 8;
  const uint32_t w_stride = D / 2, s_stride = D / BLOCK, zp_stride = (s_stride + 1) / 2;
  uint32_t tt = 0;
  float q[32];
  for (; tt + TR <= T; tt += TR) {
    for (uint32_t n = 0; n < N; n++) {
      const uint8_t* wr = w_int4 + (size_t)n * w_stride;
      const uint16_t* sr = w_scales + (size_t)n * s_stride;
      const uint8_t* zr = w_zp ? w_zp + (size_t)n * zp_stride : NULL;
      float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (uint32_t b = 0; b < s_stride; b++) {
        float scale = tso_f16_to_f32(sr[b]);
        uint32_t bd = b * BLOCK;
        decode_block(wr, bd, zr ? extract_zp(zr, b) : 0, q);
        for (uint32_t r = 0; r < TR; r++) {
          size_t xb = (size_t)(tt + r) * D + bd;
          float v[4] = {0, 0, 0, 0};
          for (int c = 0; c < 8; c++)
            for (int l = 0; l < 4; l++)
              v[l] = fmaf(load_x(x_is_f32, x, xb + 4 * c + l), q[4 * c + l], v[l]);
          float bc = (v[0] + v[1]) + (v[2] + v[3]);
          float t = bc * scale;
          sum[r] = sum[r] + t;
        }
      }
      float bv = tso_f16_to_f32(bias[n]);
      for (uint32_t r = 0; r < TR; r++) store_out(out_is_f32, out, (size_t)(tt + r) * N + n, sum[r] + bv);
    }
  }
  uint32_t m_tail = T - tt;
  if (m_tail == 0) return;
  for (uint32_t n = 0; n < N; n++) {
    const uint8_t* wr = w_int4 + (size_t)n * w_stride;
    const uint16_t* sr = w_scales + (size_t)n * s_stride;
    const uint8_t* zr = w_zp ? w_zp + (size_t)n * zp_stride : NULL;
    float accs[7] = {0, 0, 0, 0, 0, 0, 0};
    for (uint32_t b = 0; b < s_stride; b++) {
      float scale = tso_f16_to_f32(sr[b]);
      uint32_t bd = b * BLOCK;
      decode_block(wr, bd, zr ? extract_zp(zr, b) : 0, q);
      for (uint32_t ti = 0; ti < m_tail; ti++) {
        size_t xb = (size_t)(tt + ti) * D + bd;
        float a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
        for (int k = 0; k < 4; k++)
          for (int l = 0; l < 4; l++) {
            a0[l] = fmaf(load_x(x_is_f32, x, xb + 8 * k + l), q[8 * k + l], a0[l]);
            a1[l] = fmaf(load_x(x_is_f32, x, xb + 8 * k + 4 + l), q[8 * k + 4 + l], a1[l]);
          }
        float c[4];
        for (int l = 0; l < 4; l++) c[l] = a0[l] + a1[l];
        float bs = (c[0] + c[1]) + (c[2] + c[3]);
        float t = bs * scale;
        accs[ti] = accs[ti] + t;
      }
    }
    float bv = tso_f16_to_f32(bias[n]);
    for (uint32_t ti = 0; ti < m_tail; ti++)
      store_out(out_is_f32, out, (size_t)(tt + ti) * N + n, accs[ti] + bv);
  }
}

/* 32 nibbles of one block, minus zp, as eight 4-lane f32 vectors in element
 * order (int4BlockDecode, wasm_exports.zig:512-540). */
static inline void decode_block_v(const uint8_t* w_row, uint32_t block_d, uint8_t zp, __m128 q[8]) {
  const __m128i b = _mm_loadu_si128((const __m128i*)(w_row + block_d / 2));
  const __m128i m = _mm_set1_epi8(0x0F);
  const __m128i lo = _mm_and_si128(b, m);
  const __m128i hi = _mm_and_si128(_mm_srli_epi16(b, 4), m);
  const __m128i e0 = _mm_unpacklo_epi8(lo, hi); /* elements 0..15 */
  const __m128i e1 = _mm_unpackhi_epi8(lo, hi); /* elements 16..31 */
  const __m128i z = _mm_set1_epi32(zp);
  __m128i src[2] = {e0, e1};
  for (int h = 0; h < 2; h++) {
    __m128i v = src[h];
    for (int c = 0; c < 4; c++) {
      __m128i w = _mm_cvtepu8_epi32(v);
      q[h * 4 + c] = _mm_cvtepi32_ps(_mm_sub_epi32(w, z));
      v = _mm_srli_si128(v, 4);
    }
  }
}

/* (v0 + v1) + (v2 + v3) of one 4-lane vector */
static inline float hsum_pairs(__m128 v) {
  __m128 s = _mm_add_ps(v, _mm_shuffle_ps(v, v, _MM_SHUFFLE(2, 3, 0, 1)));
  return _mm_cvtss_f32(s) + _mm_cvtss_f32(_mm_movehl_ps(s, s));
}

/* Same contract and bit-identical result as tso_matmul_int4_scalar: the
 * reference's 4-lane fma4 chains are one SSE fused multiply-add per lane
 * (the Zig kernel's own vector shape), the horizontal sums keep its
 * association. */
void tso_matmul_int4(int x_is_f32, int out_is_f32, const void* x,
                     const uint8_t* w_int4, const uint16_t* w_scales, const uint8_t* w_zp,
                     const uint16_t* bias, void* out, uint32_t T, uint32_t N, uint32_t D) {
  if (!x_is_f32) {
    tso_matmul_int4_scalar(x_is_f32, out_is_f32, x, w_int4, w_scales, w_zp, bias, out, T, N, D);
    return;
  }
  const float* xf = (const float*)x;
  const uint32_t BLOCK = 32, TR = 8;
  const uint32_t w_stride = D / 2, s_stride = D / BLOCK, zp_stride = (s_stride + 1) / 2;
  uint32_t tt = 0;
  __m128 q[8];
  for (; tt + TR <= T; tt += TR) {
    for (uint32_t n = 0; n < N; n++) {
      const uint8_t* wr = w_int4 + (size_t)n * w_stride;
      const uint16_t* sr = w_scales + (size_t)n * s_stride;
      const uint8_t* zr = w_zp ? w_zp + (size_t)n * zp_stride : NULL;
      float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (uint32_t b = 0; b < s_stride; b++) {
        const float scale = tso_f16_to_f32(sr[b]);
        const uint32_t bd = b * BLOCK;
        decode_block_v(wr, bd, zr ? extract_zp(zr, b) : 0, q);
        __m128 v[8];
        for (int r = 0; r < 8; r++) v[r] = _mm_setzero_ps();
        for (int c = 0; c < 8; c++)
          for (int r = 0; r < 8; r++)
            v[r] = _mm_fmadd_ps(_mm_loadu_ps(xf + (size_t)(tt + r) * D + bd + 4 * c), q[c], v[r]);
        for (int r = 0; r < 8; r++) {
          float t = hsum_pairs(v[r]) * scale;
          sum[r] = sum[r] + t;
        }
      }
      const float bv = tso_f16_to_f32(bias[n]);
      for (uint32_t r = 0; r < TR; r++) store_out(out_is_f32, out, (size_t)(tt + r) * N + n, sum[r] + bv);
    }
  }
  const uint32_t m_tail = T - tt;
  if (m_tail == 0) return;
  for (uint32_t n = 0; n < N; n++) {
    const uint8_t* wr = w_int4 + (size_t)n * w_stride;
    const uint16_t* sr = w_scales + (size_t)n * s_stride;
    const uint8_t* zr = w_zp ? w_zp + (size_t)n * zp_stride : NULL;
    float accs[7] = {0, 0, 0, 0, 0, 0, 0};
    for (uint32_t b = 0; b < s_stride; b++) {
      const float scale = tso_f16_to_f32(sr[b]);
      const uint32_t bd = b * BLOCK;
      decode_block_v(wr, bd, zr ? extract_zp(zr, b) : 0, q);
      for (uint32_t ti = 0; ti < m_tail; ti++) {
        const float* xr = xf + (size_t)(tt + ti) * D + bd;
        __m128 a0 = _mm_setzero_ps(), a1 = _mm_setzero_ps();
        for (int k = 0; k < 4; k++) {
          a0 = _mm_fmadd_ps(_mm_loadu_ps(xr + 8 * k), q[2 * k], a0);
          a1 = _mm_fmadd_ps(_mm_loadu_ps(xr + 8 * k + 4), q[2 * k + 1], a1);
        }
        float t = hsum_pairs(_mm_add_ps(a0, a1)) * scale;
        accs[ti] = accs[ti] + t;
      }
    }
    const float bv = tso_f16_to_f32(bias[n]);
    for (uint32_t ti = 0; ti < m_tail; ti++) store_out(out_is_f32, out, (size_t)(tt + ti) * N + n, accs[ti] + bv);
  }
}

/* The dequantised operand value f32ToFp16(float(q - zp) * fp16ToF32(s)),
 * the same expression embed_lookup_int4 stores (wasm_exports.zig:1563-1570). */
void tso_dequant_int4(const uint8_t* w_int4, const uint16_t* w_scales, const uint8_t* w_zp,
                      uint16_t* out, uint32_t N, uint32_t D) {
  const uint32_t nb = D / 32, zs = (nb + 1) / 2;
  float q[32];
  for (uint32_t n = 0; n < N; n++)
    for (uint32_t b = 0; b < nb; b++) {
      float s = tso_f16_to_f32(w_scales[(size_t)n * nb + b]);
      uint8_t zp = w_zp ? extract_zp(w_zp + (size_t)n * zs, b) : 0;
      decode_block(w_int4 + (size_t)n * (D / 2), b * 32, zp, q);
      for (int i = 0; i < 32; i++) out[(size_t)n * D + b * 32 + i] = tso_f32_to_f16(q[i] * s);
    }
}

/* ------------------------------------------------------------------ */
/* SwiGLU with clamp                                                   */
/* ------------------------------------------------------------------ */

/* wasm_exports.zig:812-838: exp(x) for x <= 0 by 2^(x*log2e), floor split,
 * 5th-degree Horner polynomial with fused steps, exponent bit twiddle. */
float tso_exp_approx(float x) {
  const float LOG2_E = 1.44269504088896340736f;
  float clamped = x > -88.0f ? x : -88.0f;
  if (x != x) clamped = -88.0f; /* @max(NaN, -88) = -88 */
  float y = clamped * LOG2_E;
  int32_t iv = (int32_t)floorf(y);
  float frac = y - (float)iv;
  const float c0 = 1.000000012f, c1 = 0.693154774f, c2 = 0.240226522f;
  const float c3 = 0.055053319f, c4 = 0.009679494f, c5 = 0.001333355f;
  float p = fmaf(c5, frac, c4);
  p = fmaf(p, frac, c3);
  p = fmaf(p, frac, c2);
  p = fmaf(p, frac, c1);
  p = fmaf(p, frac, c0);
  float scale = bits_f32((uint32_t)(iv + 127) << 23);
  return p * scale;
}

/* wasm_exports.zig:844-853 */
static inline float sigmoid_approx(float x) {
  float mn = x < 0.0f ? x : 0.0f;
  float mx = x > 0.0f ? x : 0.0f;
  float neg_abs = mn - mx;
  float e = tso_exp_approx(neg_abs);
  float sig_neg = e / (1.0f + e);
  return x >= 0.0f ? 1.0f - sig_neg : sig_neg;
}

/* wasm_exports.zig:794-806 */
static inline float sigmoid_exact(float x) {
  if (x >= 0.0f) { float e = expf(-x); return 1.0f / (1.0f + e); }
  float e = expf(x);
  return e / (1.0f + e);
}

/* wasm_exports.zig:855-903 (gate = even column, up = odd column) */
void tso_swiglu_clamp_f32(const float* gate_up, float* out, uint32_t T, uint32_t D) {
  const float LIMIT = 7.0f, ALPHA = 1.702f;
  for (uint32_t t = 0; t < T; t++) {
    const float* row = gate_up + (size_t)t * 2 * D;
    float* o = out + (size_t)t * D;
    uint32_t d = 0;
    for (; d + 4 <= D; d += 4)
      for (int l = 0; l < 4; l++) {
        float g = row[2 * (d + l)], u = row[2 * (d + l) + 1];
        float gate = g < LIMIT ? g : LIMIT;           /* @min */
        float up = u < LIMIT ? u : LIMIT;
        up = up > -LIMIT ? up : -LIMIT;               /* @max */
        float scaled = gate * ALPHA;
        float sig = sigmoid_approx(scaled);
        float glu = gate * sig;
        float up1 = up + 1.0f;
        o[d + l] = up1 * glu;
      }
    for (; d < D; d++) {
      float gate = row[2 * d], up = row[2 * d + 1];
      if (gate > LIMIT) gate = LIMIT;
      if (up > LIMIT) up = LIMIT;
      if (up < -LIMIT) up = -LIMIT;
      float glu = gate * sigmoid_exact(gate * ALPHA);
      o[d] = (up + 1.0f) * glu;
    }
  }
}

/* ------------------------------------------------------------------ */
/* Elementwise / gather / scatter                                      */
/* ------------------------------------------------------------------ */

/* wasm_exports.zig:969-990 */
void tso_add_fp16(const uint16_t* a, const uint16_t* b, uint16_t* out, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) out[i] = tso_f32_to_f16(tso_f16_to_f32(a[i]) + tso_f16_to_f32(b[i]));
}

/* wasm_exports.zig:1127-1143 */
void tso_gather_f32(const float* src, const int32_t* idx, float* dst, uint32_t m, uint32_t D) {
  for (uint32_t i = 0; i < m; i++) memcpy(dst + (size_t)i * D, src + (size_t)idx[i] * D, (size_t)D * 4);
}

/* wasm_exports.zig:1027-1055: fused fma on the 4-lane body, mul+add tail. */
void tso_scatter_add_weighted_f32(float* target, const float* values, const int32_t* idx,
                                  const float* w, uint32_t m, uint32_t D) {
  for (uint32_t i = 0; i < m; i++) {
    float* tr = target + (size_t)idx[i] * D;
    const float* vr = values + (size_t)i * D;
    float wi = w[i];
    uint32_t d = 0;
    for (; d + 4 <= D; d += 4)
      for (int l = 0; l < 4; l++) tr[d + l] = fmaf(wi, vr[d + l], tr[d + l]);
    for (; d < D; d++) { float p = wi * vr[d]; tr[d] = tr[d] + p; }
  }
}

/* wasm_exports.zig:1106-1116 */
void tso_convert_fp16_to_f32(const uint16_t* src, float* dst, uint32_t n) {
  for (uint32_t i = 0; i < n; i++) dst[i] = tso_f16_to_f32(src[i]);
}

/* wasm_exports.zig:1153-1164 */
void tso_cast_f32_to_fp16_scaled(const float* src, uint16_t* dst, uint32_t n, float scale) {
  for (uint32_t i = 0; i < n; i++) dst[i] = tso_f32_to_f16(src[i] * scale);
}

/* ------------------------------------------------------------------ */
/* Banded GQA attention with sinks                                     */
/* ------------------------------------------------------------------ */

/* fp16x4ToF32x4 (math.zig:84-103) on 4 lanes */
static inline __m128 f16x4_ref(const uint16_t* p) {
  __m128i u = _mm_cvtepu16_epi32(_mm_loadl_epi64((const __m128i*)p));
  __m128i sign = _mm_slli_epi32(_mm_and_si128(u, _mm_set1_epi32(0x8000)), 16);
  __m128i rest = _mm_and_si128(u, _mm_set1_epi32(0x7fff));
  __m128i biased = _mm_add_epi32(_mm_slli_epi32(rest, 13), _mm_set1_epi32(112 << 23));
  biased = _mm_andnot_si128(_mm_cmpeq_epi32(rest, _mm_setzero_si128()), biased);
  return _mm_castsi128_ps(_mm_or_si128(sign, biased));
}

/* wasm_exports.zig:1232-1267: 4 accumulators x 4 lanes over 16-element
 * steps, then a 4-element step into a0, (a0+a1)+(a2+a3), lane sum left to
 * right, then a scalar mul+add tail. */
static inline float dot_f16(const uint16_t* a, const uint16_t* b, uint32_t n) {
  __m128 acc[4] = {_mm_setzero_ps(), _mm_setzero_ps(), _mm_setzero_ps(), _mm_setzero_ps()};
  uint32_t i = 0;
  for (; i + 16 <= n; i += 16)
    for (int u = 0; u < 4; u++) acc[u] = _mm_fmadd_ps(f16x4_ref(a + i + 4 * u), f16x4_ref(b + i + 4 * u), acc[u]);
  for (; i + 4 <= n; i += 4) acc[0] = _mm_fmadd_ps(f16x4_ref(a + i), f16x4_ref(b + i), acc[0]);
  float c[4];
  _mm_storeu_ps(c, _mm_add_ps(_mm_add_ps(acc[0], acc[1]), _mm_add_ps(acc[2], acc[3])));
  float sum = c[0] + c[1];
  sum = sum + c[2];
  sum = sum + c[3];
  for (; i < n; i++) { float p = tso_f16_to_f32(a[i]) * tso_f16_to_f32(b[i]); sum = sum + p; }
  return sum;
}

/* wasm_exports.zig:1286-1379 (banded_attention = full head range,
 * banded_attention_partial = [h_q_start, h_q_end)). */
void tso_banded_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          const float* sinks, const uint8_t* mask, uint16_t* out,
                          uint32_t T, uint32_t Hq, uint32_t Hkv, uint32_t D, uint32_t W,
                          uint32_t h_q_start, uint32_t h_q_end) {
  const uint32_t group = Hq / Hkv;
  const size_t qs = (size_t)Hq * D, ks = (size_t)Hkv * D;
  float scores[2 * 1024 + 2];
  float acc[256];
  for (uint32_t tq = 0; tq < T; tq++) {
    for (uint32_t h = h_q_start; h < h_q_end; h++) {
      const uint32_t hk = h / group;
      const size_t qb = tq * qs + (size_t)h * D;
      const uint32_t ws = tq > W ? tq - W : 0;
      const uint32_t we = (tq + W + 1 < T) ? tq + W + 1 : T;
      const uint32_t nk = we - ws;
      const float sink = sinks[h];
      float mx = sink;
      for (uint32_t j = 0; j < nk; j++) {
        uint32_t ak = ws + j;
        int valid = mask ? mask[ak] != 0 : 1;
        float s = valid ? dot_f16(q + qb, k + ak * ks + (size_t)hk * D, D) : -INFINITY;
        scores[j] = s;
        if (s > mx) mx = s;
      }
      scores[nk] = sink;
      const uint32_t total = nk + 1;
      float sv[4] = {0, 0, 0, 0};
      uint32_t i = 0;
      for (; i + 4 <= total; i += 4)
        for (int l = 0; l < 4; l++) {
          float e = tso_exp_approx(scores[i + l] - mx);
          scores[i + l] = e;
          sv[l] = sv[l] + e;
        }
      float sum = sv[0] + sv[1];
      sum = sum + sv[2];
      sum = sum + sv[3];
      for (; i < total; i++) {
        float e = expf(scores[i] - mx);
        scores[i] = e;
        sum = sum + e;
      }
      const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
      for (uint32_t d = 0; d < D; d++) acc[d] = 0.0f;
      for (uint32_t j = 0; j < nk; j++) {
        float p = scores[j] * inv;
        const uint16_t* vr = v + (ws + j) * ks + (size_t)hk * D;
        const __m128 pv4 = _mm_set1_ps(p);
        uint32_t d = 0;
        for (; d + 4 <= D; d += 4) _mm_storeu_ps(acc + d, _mm_fmadd_ps(pv4, f16x4_ref(vr + d), _mm_loadu_ps(acc + d)));
        for (; d < D; d++) { float pv = p * tso_f16_to_f32(vr[d]); acc[d] = acc[d] + pv; }
      }
      for (uint32_t d = 0; d < D; d++) out[qb + d] = tso_f32_to_f16(acc[d]);
    }
  }
}

/* ------------------------------------------------------------------ */
/* RoPE apply / embedding                                              */
/* ------------------------------------------------------------------ */

/* wasm_exports.zig:1460-1502: three fp16 roundings per output element. */
void tso_rope_apply(uint16_t* qk, const uint16_t* cos_tab, const uint16_t* sin_tab,
                    uint32_t T, uint32_t H, uint32_t D) {
  const uint32_t half = D / 2;
  for (uint32_t t = 0; t < T; t++) {
    const uint16_t* cr = cos_tab + (size_t)t * half;
    const uint16_t* sr = sin_tab + (size_t)t * half;
    for (uint32_t h = 0; h < H; h++) {
      uint16_t* x = qk + ((size_t)t * H + h) * D;
      for (uint32_t p = 0; p < half; p++) {
        float c = tso_f16_to_f32(cr[p]), s = tso_f16_to_f32(sr[p]);
        float a = tso_f16_to_f32(x[2 * p]), b = tso_f16_to_f32(x[2 * p + 1]);
        float ac = tso_f16_to_f32(tso_f32_to_f16(a * c));
        float bs = tso_f16_to_f32(tso_f32_to_f16(b * s));
        float bc = tso_f16_to_f32(tso_f32_to_f16(b * c));
        float as = tso_f16_to_f32(tso_f32_to_f16(a * s));
        x[2 * p] = tso_f32_to_f16(ac - bs);
        x[2 * p + 1] = tso_f32_to_f16(bc + as);
      }
    }
  }
}

/* wasm_exports.zig:1523-1573: out-of-range ids produce zero rows. */
void tso_embed_lookup_int4(const uint8_t* embed_int4, const uint16_t* embed_scales,
                           const uint8_t* embed_zp, const int32_t* ids, uint16_t* out,
                           uint32_t T, uint32_t V, uint32_t D) {
  const uint32_t nb = D / 32, zs = (nb + 1) / 2;
  float q[32];
  for (uint32_t t = 0; t < T; t++) {
    int32_t id = ids[t];
    uint16_t* o = out + (size_t)t * D;
    if (id < 0 || (uint32_t)id >= V) { memset(o, 0, (size_t)D * 2); continue; }
    const uint8_t* wr = embed_int4 + (size_t)id * (D / 2);
    const uint16_t* sr = embed_scales + (size_t)id * nb;
    const uint8_t* zr = embed_zp + (size_t)id * zs;
    for (uint32_t b = 0; b < nb; b++) {
      float s = tso_f16_to_f32(sr[b]);
      decode_block(wr, b * 32, extract_zp(zr, b), q);
      for (int i = 0; i < 32; i++) o[b * 32 + i] = tso_f32_to_f16(q[i] * s);
    }
  }
}
