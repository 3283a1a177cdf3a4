/*
 * htp_oracle.c — CPU restatement of the reference linear-operator arithmetic.
 * TEST INFRASTRUCTURE ONLY (see htp_oracle.h).  Build with -ffp-contract=off.
 *
 * Reference files cited below are paths inside destined555/htp-ops-lib-sd.cpp.
 */
#include "htp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

int orc_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------------------------------------------------ */
/* Seeded generators                                                        */
/* ------------------------------------------------------------------------ */

uint64_t orc_splitmix64(uint64_t *state) {
  uint64_t z = (*state += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

/* uniform double in [0, 1) with 53 random bits */
static double unit_double(uint64_t *s) { return (double)(orc_splitmix64(s) >> 11) * 0x1.0p-53; }

void orc_fill_normal(float *dst, size_t count, double sigma, double outlier_p, double outlier_scale,
                     uint64_t seed) {
  uint64_t s = seed;
  for (size_t i = 0; i < count; i += 2) {
    /* Box-Muller on FP64: u1 in (0,1], u2 in [0,1) */
    const double u1 = 1.0 - unit_double(&s);
    const double u2 = unit_double(&s);
    const double r = sqrt(-2.0 * log(u1));
    const double z[2] = {r * cos(2.0 * M_PI * u2), r * sin(2.0 * M_PI * u2)};
    for (int j = 0; j < 2 && i + j < count; ++j) {
      double v = sigma * z[j];
      if (outlier_p > 0.0 && unit_double(&s) < outlier_p) v *= outlier_scale;
      dst[i + j] = (float)v;
    }
  }
}

void orc_fill_uniform(float *dst, size_t count, double lo, double hi, uint64_t seed) {
  uint64_t s = seed;
  for (size_t i = 0; i < count; ++i) dst[i] = (float)(lo + (hi - lo) * unit_double(&s));
}

void orc_fill_int8(int8_t *dst, size_t count, uint64_t seed) {
  uint64_t s = seed;
  for (size_t i = 0; i < count; ++i) dst[i] = (int8_t)((int)(orc_splitmix64(&s) % 255u) - 127);
}

void orc_fill_f16_normal(uint16_t *dst, size_t count, double sigma, uint64_t seed) {
  float *tmp = (float *)malloc(count * sizeof(float));
  orc_fill_normal(tmp, count, sigma, 0.0, 1.0, seed);
  for (size_t i = 0; i < count; ++i) dst[i] = orc_f32_to_f16(tmp[i]);
  free(tmp);
}

/* ------------------------------------------------------------------------ */
/* FP16 conversion (IEEE binary16, round to nearest even)                   */
/* ------------------------------------------------------------------------ */

uint16_t orc_f32_to_f16(float x) {
  _Float16 h = (_Float16)x;
  uint16_t bits;
  memcpy(&bits, &h, 2);
  return bits;
}

float orc_f16_to_f32(uint16_t bits) {
  _Float16 h;
  memcpy(&h, &bits, 2);
  return (float)h;
}

static inline uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float bits_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ------------------------------------------------------------------------ */
/* Layouts                                                                  */
/* ------------------------------------------------------------------------ */

/* Weight region of the constants blob: groups of 64 output columns, each a
 * run of K/32 slices of 2048 bytes; a slice holds two 32-column halves of
 * 1024 bytes; inside a half, byte (n%32)*4 + k%4 of row (k%32)/4 (128 bytes).
 * linear_w8a8.c:453 (group base n0*k), :487 (slice t*2048, "weight.b ... :deep"),
 * study_dsp.c:79-84 (tile (t*banks+h)*1024, (k/4)*128 + n*4 + k%4). */
size_t orc_deep_offset(int k_total, int n, int k) {
  return (size_t)(n / 64) * 64u * (size_t)k_total + (size_t)(k / 32) * 2048u +
         (size_t)((n % 64) / 32) * 1024u + (size_t)((k % 32) / 4) * 128u + (size_t)(n % 32) * 4u +
         (size_t)(k % 4);
}

size_t orc_w8a8_blob_bytes(int k, int n) {
  return 128u + (size_t)k * n + (size_t)n * 8u + (size_t)k * 4u;
}

void orc_w8a8_pack(uint8_t *blob, const int8_t *w_nk, const float *sw, const float *inverse,
                   int k, int n, uint64_t signature) {
  const size_t bytes = orc_w8a8_blob_bytes(k, n);
  memset(blob, 0, 128);
  uint32_t *h = (uint32_t *)blob;
  h[0] = 0x38574d48u; /* magic "HMW8" */
  h[1] = 1;           /* version */
  h[2] = (uint32_t)k;
  h[3] = (uint32_t)n;
  h[4] = 128;                                 /* weight_offset */
  h[5] = 128u + (uint32_t)((size_t)k * n);    /* scale_offset */
  h[6] = h[5] + 4u * (uint32_t)n;             /* sum_offset */
  h[7] = h[6] + 4u * (uint32_t)n;             /* inverse_offset */
  h[8] = (uint32_t)bytes;                     /* bytes */
  memcpy(blob + 40, &signature, 8);           /* original_f16_signature */
  uint8_t *weights = blob + 128;
  float *scales = (float *)(blob + h[5]);
  int32_t *sums = (int32_t *)(blob + h[6]);
  float *inv = (float *)(blob + h[7]);
  for (int c = 0; c < n; ++c) {
    int32_t sum = 0;
    for (int r = 0; r < k; ++r) {
      const int8_t v = w_nk[(size_t)c * k + r];
      weights[orc_deep_offset(k, c, r)] = (uint8_t)v;
      sum += v;
    }
    sums[c] = sum;
    scales[c] = sw[c];
  }
  for (int r = 0; r < k; ++r) inv[r] = inverse ? inverse[r] : 1.0f;
}

void orc_w8a8_unpack_weight(int8_t *w_nk, const uint8_t *blob, int k, int n) {
  const uint32_t *h = (const uint32_t *)blob;
  const uint8_t *weights = blob + h[4];
#pragma omp parallel for schedule(static)
  for (int c = 0; c < n; ++c)
    for (int r = 0; r < k; ++r) w_nk[(size_t)c * k + r] = (int8_t)weights[orc_deep_offset(k, c, r)];
}

/* FP16 permuted weight: 32x32 tiles, tile (n/32)*(K/32) + k/32 of 1024
 * elements; inside, element ((k%32) & ~1)*32 + (n%32)*2 + (k & 1)
 * (src/host/test.c:548-556, mat_mul.c:994 chunk base nc*K). */
size_t orc_f16_perm_offset(int k_total, int k, int n) {
  const size_t tile = (size_t)(n / 32) * (size_t)(k_total / 32) + (size_t)(k / 32);
  return tile * 1024u + (size_t)((k % 32) & ~1) * 32u + (size_t)(n % 32) * 2u + (size_t)(k & 1);
}

void orc_f16_pack_permuted(uint16_t *dst, const uint16_t *w_kn, int k, int n) {
  for (int r = 0; r < k; ++r)
    for (int c = 0; c < n; ++c) dst[orc_f16_perm_offset(k, r, c)] = w_kn[(size_t)r * n + c];
}

/* Compact CM activation tiles: tile (m/64)*64*K + (k/32)*2048, row-major
 * 64 x 32 bytes inside (linear_w8a8.c:117, 281). */
size_t orc_cm_offset(int k_total, int m, int k) {
  return (size_t)(m / 64) * 64u * (size_t)k_total + (size_t)(k / 32) * 2048u +
         (size_t)(m % 64) * 32u + (size_t)(k % 32);
}

/* ------------------------------------------------------------------------ */
/* W8A8                                                                     */
/* ------------------------------------------------------------------------ */

/* One row of linear_w8a8.c:65-118 (prepare_tile_impl): x' = x*inverse,
 * absmax, scale = fmaxf(absmax/127, 1e-12f) (row_scale :34-40), s = 1/scale
 * (:106), then quantize_scaled (:42-59): u = x'*s + 128 (two IEEE roundings),
 * clamp to [1,255] by integer max/min on the IEEE bits, round half to even. */
static float quantize_row(uint8_t *codes, const float *x, const float *inverse, int k,
                          float *scratch) {
  float absmax = 0.0f;
  for (int c = 0; c < k; ++c) {
    const float v = inverse ? x[c] * inverse[c] : x[c];
    scratch[c] = v;
    const float a = fabsf(v);
    absmax = fmaxf(absmax, a);
  }
  const float scale = fmaxf(absmax / 127.0f, 1e-12f);
  const float s = 1.0f / scale;
  for (int c = 0; c < k; ++c) {
    const float t = scratch[c] * s;
    const float u = t + 128.0f;
    int32_t b = (int32_t)f32_bits(u);
    if (b < (int32_t)0x3f800000) b = (int32_t)0x3f800000; /* 1.0f */
    if (b > (int32_t)0x437f0000) b = (int32_t)0x437f0000; /* 255.0f */
    codes[c] = (uint8_t)rintf(bits_f32((uint32_t)b));     /* RNE in default mode */
  }
  return scale;
}

void orc_quantize_rows(uint8_t *codes, float *scales, const float *x, const float *inverse,
                       int m, int k) {
#pragma omp parallel
  {
    float *scratch = (float *)malloc((size_t)k * sizeof(float));
#pragma omp for schedule(static)
    for (int r = 0; r < m; ++r)
      scales[r] = quantize_row(codes + (size_t)r * k, x + (size_t)r * k, inverse, k, scratch);
    free(scratch);
  }
}

static inline int32_t dot_u8_s8(const uint8_t *a, const int8_t *b, int k) {
  int32_t acc = 0;
  for (int i = 0; i < k; ++i) acc += (int32_t)a[i] * (int32_t)b[i];
  return acc;
}

void orc_w8a8_accumulate(int32_t *acc, const uint8_t *codes, const int8_t *w_nk, int m, int k,
                         int n) {
#pragma omp parallel for collapse(2) schedule(static)
  for (int r = 0; r < m; ++r)
    for (int c = 0; c < n; ++c)
      acc[(size_t)r * n + c] = dot_u8_s8(codes + (size_t)r * k, w_nk + (size_t)c * k, k);
}

/* Optional epilogue shared by both operators (mat_mul.c:788-826 and
 * :864-882): GELU(tanh) as x*sigmoid(1.5957691216057308*(x + 0.044715 x^3)),
 * QuickGELU as x*sigmoid(1.702 x).  The sigmoid keeps the reference's stable
 * structure e = 2^max(-|z|*log2(e), -126), inv = 1/(1+e),
 * sigma = z < 0 ? e*inv : inv, with libm exp2f and an exact division in place
 * of the HVX polynomial and Newton steps. */
float orc_epilogue_activation(float x, int mode) {
  if (mode != 1 && mode != 2) return x;
  float z;
  if (mode == 1) {
    const float cubic = (x * x) * x;
    z = x + cubic * 0.044715f;
    z = z * 1.5957691216057308f;
  } else {
    z = x * 1.702f;
  }
  float arg = fabsf(z) * -1.4426950408889634f;
  arg = fmaxf(arg, -126.0f);
  const float e = exp2f(arg);
  const float inv = 1.0f / (e + 1.0f);
  const float sig = z < 0.0f ? e * inv : inv;
  return x * sig;
}

static inline void store_out(float *out, int mode, int channels, int nrows, int r, int c, int n,
                             float v) {
  if (mode == 3) {
    if (c < channels) out[(size_t)c * nrows + r] = v; /* mat_mul.c:847-858 */
  } else {
    out[(size_t)r * n + c] = v;
  }
}

void orc_w8a8_linear_rows(float *out, const float *x, const uint8_t *blob, const float *bias,
                          int m, int k, int n, int channels, int mode, const int32_t *rows,
                          int nrows, uint8_t *codes_out, float *scales_out,
                          int32_t *signed_acc_out) {
  (void)m;
  const uint32_t *h = (const uint32_t *)blob;
  const float *sw = (const float *)(blob + h[5]);
  const int32_t *sums = (const int32_t *)(blob + h[6]);
  const float *inverse = (const float *)(blob + h[7]);
  int8_t *w = (int8_t *)malloc((size_t)k * n);
  orc_w8a8_unpack_weight(w, blob, k, n);
#pragma omp parallel
  {
    float *scratch = (float *)malloc((size_t)k * sizeof(float));
    uint8_t *codes = (uint8_t *)malloc((size_t)k);
#pragma omp for schedule(dynamic, 1)
    for (int i = 0; i < nrows; ++i) {
      const int row = rows ? rows[i] : i;
      const float rs = quantize_row(codes, x + (size_t)row * k, inverse, k, scratch);
      if (codes_out) memcpy(codes_out + (size_t)i * k, codes, (size_t)k);
      if (scales_out) scales_out[i] = rs;
      for (int c = 0; c < n; ++c) {
        const int32_t acc = dot_u8_s8(codes, w + (size_t)c * k, k);
        /* zero-point correction acc - (sum << 7) (linear_w8a8.c:159, 168),
         * done in wrapping 32-bit arithmetic like the HVX word ops */
        const int32_t y = (int32_t)((uint32_t)acc - ((uint32_t)sums[c] << 7));
        if (signed_acc_out) signed_acc_out[(size_t)i * n + c] = y;
        float v = (float)y;   /* Q6_Vsf_equals_Vw: nearest even */
        v = v * sw[c];        /* column scale first (:174) */
        v = v * rs;           /* then the row scale (:176) */
        if (bias) v = v + bias[c];
        v = orc_epilogue_activation(v, mode);
        store_out(out, mode, channels, nrows, i, c, n, v);
      }
    }
    free(codes);
    free(scratch);
  }
  free(w);
}

/* ------------------------------------------------------------------------ */
/* FP16 GEMM + epilogue                                                     */
/* ------------------------------------------------------------------------ */

/* mat_mul.c:937-1044: activation rounded to FP16 (:114-148), FP16 x FP16
 * products accumulated over the whole K (:724-748; K is never split,
 * f16_gemm_plan.h:11-12), optional bias then activation (:864-882) or the
 * cropped channel-major store (:830-862). */
void orc_f16_linear_rows(float *out, const float *x, const uint16_t *wperm, const float *bias,
                         int m, int k, int n, int channels, int mode, int round_acc_f16,
                         const int32_t *rows, int nrows) {
  (void)m;
  /* weights as FP32 [n][k] */
  float *w = (float *)malloc((size_t)k * n * sizeof(float));
#pragma omp parallel for schedule(static)
  for (int c = 0; c < n; ++c)
    for (int r = 0; r < k; ++r)
      w[(size_t)c * k + r] = orc_f16_to_f32(wperm[orc_f16_perm_offset(k, r, c)]);
#pragma omp parallel
  {
    float *a = (float *)malloc((size_t)k * sizeof(float));
#pragma omp for schedule(dynamic, 1)
    for (int i = 0; i < nrows; ++i) {
      const int row = rows ? rows[i] : i;
      for (int r = 0; r < k; ++r) a[r] = orc_f16_to_f32(orc_f32_to_f16(x[(size_t)row * k + r]));
      for (int c = 0; c < n; ++c) {
        const float *wc = w + (size_t)c * k;
        float acc = 0.0f;
        for (int r = 0; r < k; ++r) acc += a[r] * wc[r]; /* products exact in FP32 */
        if (round_acc_f16) acc = orc_f16_to_f32(orc_f32_to_f16(acc));
        float v = acc;
        if (bias) v = v + bias[c];
        v = orc_epilogue_activation(v, mode);
        store_out(out, mode, channels, nrows, i, c, n, v);
      }
    }
    free(a);
  }
  free(w);
}

/* Follows export_plane_tile (linear_w8a8.c:209-227): per half, a flat byte
 * counter walks plane 0..3, each `rows`*32 bytes; byte `flat` goes to output
 * row flat/128 of the tile, byte flat%128 of the half's 128-byte span.  The
 * plane bytes come from the HMX readout (read_int32, :130-138), whose plane p
 * holds byte p of each 32-bit accumulator at (row, column) offset row*32+col. */
void orc_w8a8_planes(uint8_t *out, const int32_t *acc, int m, int n) {
  for (int t = 0; t * 64 < m; ++t) {
    const int rows = m - t * 64 < 64 ? m - t * 64 : 64;
    for (int g = 0; g < n / 64; ++g) {
      for (int h = 0; h < 2; ++h) {
        size_t flat = 0;
        for (int p = 0; p < 4; ++p) {
          for (int r = 0; r < rows; ++r) {
            for (int c = 0; c < 32; ++c, ++flat) {
              const uint32_t v = (uint32_t)acc[(size_t)(t * 64 + r) * n + g * 64 + h * 32 + c];
              const size_t dst_row = (size_t)t * 64 + flat / 128;
              out[(dst_row * n + (size_t)g * 64 + h * 32) * 4 + flat % 128] = (uint8_t)(v >> (8 * p));
            }
          }
        }
      }
    }
  }
}

/* Follows conv_gather_worker (mat_mul.c:2230-2290), general branch :2281-2286:
 * for output position t and K column col (kx = (col%kw)*dx, ky =
 * ((col/kw)%kh)*dy, ci = col/(kw*kh)), x = (t%ow)*sx - px + kx and
 * y = (t/ow)*sy - py + ky in the upsampled image; the value is
 * input[ci][y/up][x/up] inside it and 0 outside or for ci >= ic. */
void orc_conv_im2col(float *a, const float *x, const int32_t *prm, int b) {
  const int iw = prm[0], ih = prm[1], ic = prm[2], ow = prm[5], oh = prm[6], kw = prm[7], kh = prm[8];
  const int sx = prm[9], sy = prm[10], px = prm[11], py = prm[12], dx = prm[13], dy = prm[14], kp = prm[15];
  const int up = prm[17];
  const float *in = x + (size_t)b * iw * ih * ic;
#pragma omp parallel for schedule(static)
  for (int t = 0; t < ow * oh; ++t) {
    for (int col = 0; col < kp; ++col) {
      const int kx = (col % kw) * dx, ky = ((col / kw) % kh) * dy, ci = col / (kw * kh);
      const int xx = (t % ow) * sx - px + kx, yy = (t / ow) * sy - py + ky;
      float v = 0.0f;
      if (ci < ic && xx >= 0 && xx < iw * up && yy >= 0 && yy < ih * up)
        v = in[((size_t)ci * ih + yy / up) * iw + xx / up];
      a[(size_t)t * kp + col] = v;
    }
  }
}

/* hmx_conv2d_nchw_f16 (mat_mul.c:2291-2343): per batch, im2col then the FP16
 * GEMM with the mode-3 (bias + channel-major) epilogue over oc channels. */
void orc_conv2d_nchw_f16(float *out, const float *x, const uint16_t *wperm, const float *bias,
                         const int32_t *prm, int round_acc_f16) {
  const int oc = prm[3], batch = prm[4], ow = prm[5], oh = prm[6], kp = prm[15], np = prm[16];
  const int spatial = ow * oh;
  float *a = (float *)malloc((size_t)spatial * kp * sizeof(float));
  for (int b = 0; b < batch; ++b) {
    orc_conv_im2col(a, x, prm, b);
    orc_f16_linear_rows(out + (size_t)b * oc * spatial, a, wperm, bias, spatial, kp, np, oc, 3, round_acc_f16,
                        NULL, spatial);
  }
  free(a);
}

/* ------------------------------------------------------------------------ */
/* Opcodes 2-4: ggml-block weights (mat_mul.c:246-430, 1601-1874)           */
/* ------------------------------------------------------------------------ */

/* IQ4_NL levels (iq4_nl_to_fp16_lut, mat_mul.c:34-37: the table holds its 16
 * entries at the even half-word positions that vlut16 reads). */
static const int8_t kIq4nlLevels[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                        1,    13,   25,  38,  53,  69,  89,  113};

size_t orc_qk0_block_bytes(int type) {
  switch (type) {
    case ORC_GGML_Q4_0:
    case ORC_GGML_IQ4_NL: return 16 + 128; /* my_block_q4_0 (quants.h:16-19) */
    case ORC_GGML_Q8_0: return 16 + 256;   /* my_block_q8_0 (quants.h:28-31) */
    default: return 0;
  }
}

/* Element e of a super-block, following the per-block body of
 * dequantize_permuted_weight_q4_0_to_fp16_hvx_task (mat_mul.c:389-424) and
 * ..._q8_0_... (:488-525).  Q4: vlut16 on the low nibbles (v = 0: even bytes,
 * v = 1: odd bytes) and on the bytes shifted right by 4 (v = 2, 3); the scale
 * vectors hold scales[2v] for lanes 0..31 and scales[2v+1] for 32..63 (the
 * vlut16 of the {0,2 | 1,3} index pattern over the unpacked scales).  Q8:
 * vunpack keeps byte order, so element e is byte e. */
uint16_t orc_qk0_element(const uint8_t *block, int type, int e) {
  uint16_t sbits;
  memcpy(&sbits, block + 2 * (e / 32), 2);
  const float scale = orc_f16_to_f32(sbits);
  const uint8_t *q = block + 16;
  float level;
  if (type == ORC_GGML_Q8_0) {
    level = (float)(int8_t)q[e];
  } else {
    const int v = e / 64, i = e % 64;
    const uint8_t byte = q[2 * i + (v & 1)];
    const int nib = v < 2 ? (byte & 15) : (byte >> 4);
    level = type == ORC_GGML_IQ4_NL ? (float)kIq4nlLevels[nib] : (float)(nib - 8);
  }
  /* |level| <= 128 and an 11-bit significand: the product is exact in FP32,
     so one rounding to FP16 remains */
  return orc_f32_to_f16(level * scale);
}

/* The dequantised stream is the packed FP16 weight itself. */
static void qk0_stream(uint16_t *perm, const uint8_t *src, int type, int k, int n) {
  const size_t bb = orc_qk0_block_bytes(type);
  const size_t blocks = (size_t)k * (size_t)n / 256u;
#pragma omp parallel for schedule(static)
  for (size_t b = 0; b < blocks; ++b)
    for (int e = 0; e < 256; ++e) perm[b * 256u + (size_t)e] = orc_qk0_element(src + b * bb, type, e);
}

void orc_qk0_dequant(uint16_t *w_nk, const uint8_t *src, int type, int k, int n) {
  uint16_t *perm = (uint16_t *)malloc((size_t)k * n * 2u);
  qk0_stream(perm, src, type, k, n);
  for (int c = 0; c < n; ++c)
    for (int r = 0; r < k; ++r) w_nk[(size_t)c * k + r] = perm[orc_f16_perm_offset(k, r, c)];
  free(perm);
}

/* (k, n) of packed FP16 position f: the inverse of orc_f16_perm_offset. */
static void perm_position(size_t f, int k_total, int *k, int *n) {
  const size_t tile = f / 1024u, o = f % 1024u;
  const int kt = (int)(tile % (size_t)(k_total / 32)), nt = (int)(tile / (size_t)(k_total / 32));
  *k = kt * 32 + (int)(o / 64u) * 2 + (int)(o & 1u);
  *n = nt * 32 + (int)((o % 64u) / 2u);
}

void orc_qk0_quantize(uint8_t *dst, const float *w_kn, int type, int k, int n) {
  const size_t bb = orc_qk0_block_bytes(type);
  const size_t blocks = (size_t)k * (size_t)n / 256u;
  for (size_t b = 0; b < blocks; ++b) {
    uint8_t *blk = dst + b * bb;
    memset(blk, 0, bb);
    for (int g = 0; g < 8; ++g) {
      float vals[32], mx = 0.0f;
      for (int j = 0; j < 32; ++j) {
        int r, c;
        perm_position(b * 256u + (size_t)(g * 32 + j), k, &r, &c);
        vals[j] = w_kn[(size_t)r * n + c];
        if (fabsf(vals[j]) > fabsf(mx)) mx = vals[j];
      }
      /* the extreme value maps onto the most negative level exactly */
      const float lo = type == ORC_GGML_Q4_0 ? -8.0f : -127.0f;
      const uint16_t dbits = orc_f32_to_f16(type == ORC_GGML_Q8_0 ? fabsf(mx) / 127.0f : mx / lo);
      memcpy(blk + 2 * g, &dbits, 2);
      const float d = orc_f16_to_f32(dbits);
      for (int j = 0; j < 32; ++j) {
        const int e = g * 32 + j;
        int code;
        if (type == ORC_GGML_IQ4_NL) {
          code = 0;
          for (int t = 1; t < 16; ++t)
            if (fabsf(vals[j] - d * kIq4nlLevels[t]) < fabsf(vals[j] - d * kIq4nlLevels[code])) code = t;
        } else {
          const float r = d != 0.0f ? nearbyintf(vals[j] / d) : 0.0f;
          const float hi = type == ORC_GGML_Q4_0 ? 7.0f : 127.0f;
          code = (int)fminf(fmaxf(r, type == ORC_GGML_Q4_0 ? -8.0f : -127.0f), hi);
          if (type == ORC_GGML_Q4_0) code += 8;
        }
        if (type == ORC_GGML_Q8_0) {
          blk[16 + e] = (uint8_t)(int8_t)code;
        } else {
          const int v = e / 64, i = e % 64;
          uint8_t *byte = blk + 16 + 2 * i + (v & 1);
          *byte |= (uint8_t)(v < 2 ? code : code << 4);
        }
      }
    }
  }
}

void orc_qk0_linear_rows(float *out, const float *x, const uint8_t *src, int type, int m, int k, int n,
                         int round_acc_f16, const int32_t *rows, int nrows) {
  uint16_t *perm = (uint16_t *)malloc((size_t)k * n * 2u);
  qk0_stream(perm, src, type, k, n);
  orc_f16_linear_rows(out, x, perm, NULL, m, k, n, n, 0, round_acc_f16, rows, nrows);
  free(perm);
}

/* epilogue_activation (mat_mul.c:788-826): z = x (SiLU), 1.702x (QuickGELU) or
 * 1.5957691216057308*(x + 0.044715x^3) (GELU); x*sigmoid(z) with the stable
 * split e = 2^(-|z| log2 e), sigmoid = z < 0 ? e/(1+e) : 1/(1+e). */
float orc_activation(float x, int mode) {
  if (mode != 1 && mode != 2 && mode != 4 && mode != 5) return x;
  float z = x;
  if (mode == 1) z = x + (x * x * x) * 0.044715f;
  z = z * (mode == 1 ? 1.5957691216057308f : (mode == 4 || mode == 5) ? 1.0f : 1.702f);
  float neg = fabsf(z) * -1.4426950408889634f;
  if (neg < -126.0f) neg = -126.0f;
  const float e = exp2f(neg);
  const float inv = 1.0f / (e + 1.0f);
  const float sig = z < 0.0f ? e * inv : inv;
  return x * sig;
}

/* Mean and 1/sqrt(var + eps) of n values as the reference forms them: sums
 * in double, mean and the scale as FP32 (mat_mul.c:2397-2408). */
static void aux_stats(const float *x, long n, int center, float eps, float *mean, float *inv) {
  double s = 0.0;
  if (center)
    for (long i = 0; i < n; ++i) s += x[i];
  const float m = center ? (float)(s / n) : 0.0f;
  double q = 0.0;
  for (long i = 0; i < n; ++i) {
    const float d = x[i] - m;
    q += (double)d * d;
  }
  *mean = m;
  *inv = 1.0f / sqrtf((float)(q / n + eps));
}

/* Follows model_aux_worker (mat_mul.c:2356-2470) mode by mode. */
void orc_model_aux(float *out, const float *x, const float *w, const float *b, const int32_t *prm, float eps) {
  const int mode = prm[0], count = prm[1], width = prm[2], channels = prm[3], spatial = prm[4];
  const int groups = prm[5], batch = prm[6], other = prm[7], act = prm[8];
  if (mode <= 2 || mode == 9) {
    const long n = mode == 2 ? (long)spatial * (channels / groups) : width;
    const long tasks = mode == 2 ? (long)groups * batch : count / width;
    for (long t = 0; t < tasks; ++t) {
      const long off = t * n;
      float mean, inv;
      aux_stats(x + off, n, mode != 1, eps, &mean, &inv);
      for (long i = 0; i < n; ++i) {
        float v = (x[off + i] - mean) * inv;
        if (mode == 2) {
          const int ch = (int)(((off + i) / spatial) % channels);
          if (w) v = v * w[ch];
          if (b) v = v + b[ch];
        } else if (mode == 9) {
          const long pb = other == width ? 0 : t / spatial;
          v = v + v * w[pb * width + i];
          v = v + b[pb * width + i];
        } else {
          if (w) v = v * w[i];
          if (b) v = v + b[i];
        }
        if (act) v = orc_activation(v, 4);
        out[off + i] = v;
      }
    }
  } else if (mode == 8) {
    for (int bb = 0; bb < batch; ++bb)
      for (int r = 0; r < width; ++r)
        for (int c = 0; c < spatial; ++c)
          out[((long)bb * spatial + c) * width + r] = x[((long)bb * width + r) * spatial + c];
  } else if (mode == 11) {
    const int dim = width, heads = channels;
    for (int bb = 0; bb < batch; ++bb)
      for (int tok = 0; tok < spatial; ++tok) {
        const float *pe = w + ((long)(groups == 1 ? 0 : bb) * spatial + tok) * dim * 2;
        for (int h = 0; h < heads; ++h) {
          const float *xi = x + (((long)bb * spatial + tok) * heads + h) * dim;
          float *o = out + (((long)bb * heads + h) * spatial + tok) * dim;
          for (int e = 0; e < dim; e += 2) {
            const float *m = pe + 2 * e;
            o[e] = xi[e] * m[0] + xi[e + 1] * m[1];
            o[e + 1] = xi[e + 1] * m[3] + xi[e] * m[2];
          }
        }
      }
  } else if (mode == 12) {
    for (long i = 0; i < count; ++i) {
      const long row = i / width, col = i % width;
      const float *a = x + row * channels + col;
      const float gate = act ? a[0] : a[width], up = act ? a[width] : a[0];
      out[i] = orc_activation(gate, 5) * up;
    }
  } else if (mode == 13) {
    const int att = groups, ow = width + att;
    for (long t = 0; t < (long)spatial * batch; ++t) {
      for (int i = 0; i < att; ++i) out[t * ow + i] = w[t * att + i];
      const float *a = x + t * channels;
      for (int i = 0; i < width; ++i) {
        const float gate = act ? a[i] : a[i + width], up = act ? a[i + width] : a[i];
        out[t * ow + att + i] = orc_activation(gate, 5) * up;
      }
    }
  } else if (mode == 10) {
    for (long i = 0; i < count; ++i) {
      const int ch = (int)(i % width);
      const long bb = i / ((long)width * spatial), pb = other == width ? 0 : bb;
      out[i] = x[i] * w[pb * width + ch] + b[i];
    }
  } else if (mode == 3 || mode == 4) {
    for (long i = 0; i < count; ++i) out[i] = mode == 3 ? x[i] + w[i % other] : x[i] * w[i % other];
  } else {
    const int am = mode == 5 ? 4 : mode == 6 ? 1 : 2;
    for (long i = 0; i < count; ++i) out[i] = orc_activation(x[i], am);
  }
}
