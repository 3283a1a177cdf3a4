/*
 * htp_oracle — CPU restatement of the reference library's linear-operator
 * arithmetic (W8A8 opcode 15, packed FP16 GEMM + epilogue opcodes 1/16, the
 * ggml-block dequantising GEMMs of opcodes 2-4, convolution opcode 17 and the
 * model auxiliaries of opcode 19).
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in libhtp_ops_b200.so links or calls this
 * code; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * use it, as the checker.
 *
 * Parity pinning (what this restatement is checked against):
 *  - integer semantics (UINT8 x INT8 -> exact INT32, zero-point-128
 *    correction, HMX "deep" N64 weight layout, CM activation tiles, FP16
 *    crouton layout) against the known-answer cases of the reference's HMX
 *    probe (tests/hmx-probe/integer_tests.c:79-134, study_data.h:1-21,
 *    study_dsp.c:70-86) and its host layout demo (src/host/test.c:545-556);
 *  - the wire ABI and the planner against the reference headers/test compiled
 *    here (oracle/_ref);
 *  - FP32 arithmetic: IEEE single precision with no contraction
 *    (-ffp-contract=off, as the reference builds linear_w8a8.c,
 *    CMakeLists.txt:97-98).  The reference executes these steps in HVX QFloat,
 *    whose ulp-level rounding is undocumented and cannot run here, so the FP32
 *    steps are pinned only by this restatement ("parity unpinned" at the ulp
 *    level of QFloat; within the output tolerances otherwise).
 */
#ifndef HTP_ORACLE_H
#define HTP_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded synthetic inputs (splitmix64; Box-Muller on FP64) ---------- */
uint64_t orc_splitmix64(uint64_t *state);
/* N(0, sigma) rounded to FP32; each element independently multiplied by
 * outlier_scale with probability outlier_p. */
void orc_fill_normal(float *dst, size_t count, double sigma, double outlier_p,
                     double outlier_scale, uint64_t seed);
void orc_fill_uniform(float *dst, size_t count, double lo, double hi, uint64_t seed);
/* uniform integers in [-127, 127] */
void orc_fill_int8(int8_t *dst, size_t count, uint64_t seed);
/* FP16 bit patterns of N(0, sigma) */
void orc_fill_f16_normal(uint16_t *dst, size_t count, double sigma, uint64_t seed);

/* ---- FP16 helpers ------------------------------------------------------ */
uint16_t orc_f32_to_f16(float x); /* round to nearest even */
float orc_f16_to_f32(uint16_t h);

/* ---- layouts ------------------------------------------------------------ */
/* Byte offset of W[n][k] inside the weight region of a constants blob
 * (HMX deep N64 layout; linear_w8a8.c:453,482,487; study_dsp.c:79-84). */
size_t orc_deep_offset(int k_total, int n, int k);
size_t orc_w8a8_blob_bytes(int k, int n);
/* Build a constants blob from row-major w[n][k], sw[n], inverse[k] (NULL = 1).
 * sums[n] = sum_k w[n][k]. */
void orc_w8a8_pack(uint8_t *blob, const int8_t *w_nk, const float *sw, const float *inverse,
                   int k, int n, uint64_t signature);
void orc_w8a8_unpack_weight(int8_t *w_nk, const uint8_t *blob, int k, int n);
/* Offset (in FP16 elements) of W16[k][n] in the permuted layout
 * (src/host/test.c:548-556). */
size_t orc_f16_perm_offset(int k_total, int k, int n);
void orc_f16_pack_permuted(uint16_t *dst, const uint16_t *w_kn, int k, int n);
/* Offset of activation code (m,k) in the compact CM tiles (linear_w8a8.c:117,281). */
size_t orc_cm_offset(int k_total, int m, int k);

/* ---- W8A8 (reference: linear_w8a8.c) ------------------------------------ */
/* Per-row quantisation (linear_w8a8.c:34-128).  codes: UINT8 [m][k] in [1,255]
 * (zero point 128); scales: [m]. */
void orc_quantize_rows(uint8_t *codes, float *scales, const float *x, const float *inverse,
                       int m, int k);
/* acc[m][n] = sum_k code[m][k] * w[n][k]  (UINT8 x INT8 -> INT32, a4). */
void orc_w8a8_accumulate(int32_t *acc, const uint8_t *codes, const int8_t *w_nk,
                         int m, int k, int n);
/* CPU-epilogue export (reference: linear_w8a8.c:205-227, read_int32 :130-138):
 * the unsigned-code accumulators acc[m][n] as byte planes in the output
 * tensor's bytes.  out: m*n*4 bytes (the FP32 output tensor).  For every 64-row
 * tile (rows = its valid rows), 64-column group g and half h: the half's four
 * 64x32-byte planes (byte p of each accumulator, row-major) are concatenated
 * and written 128 bytes per output row into columns g*64+h*32 .. +31. */
void orc_w8a8_planes(uint8_t *out, const int32_t *acc, int m, int n);
/* Full operator on a subset of rows.  rows: `nrows` row indices of x (NULL =
 * rows 0..m-1 with nrows = m).  out: [nrows][n] for mode 0-2; for mode 3
 * [channels][nrows].  bias may be NULL.  Also returns codes/scales/signed
 * accumulators of those rows when the pointers are non-NULL. */
void orc_w8a8_linear_rows(float *out, const float *x, const uint8_t *blob, const float *bias,
                          int m, int k, int n, int channels, int mode,
                          const int32_t *rows, int nrows,
                          uint8_t *codes_out, float *scales_out, int32_t *signed_acc_out);

/* ---- FP16 GEMM + epilogue (reference: mat_mul.c:724-1049) --------------- */
float orc_epilogue_activation(float x, int mode);
/* out rows as above.  round_acc_f16 != 0 rounds each accumulator to FP16
 * before the epilogue (HMX "cvt.hf = acc", hmx_utils.h:34-40). */
void orc_f16_linear_rows(float *out, const float *x, const uint16_t *wperm, const float *bias,
                         int m, int k, int n, int channels, int mode, int round_acc_f16,
                         const int32_t *rows, int nrows);

/* ---- opcode 17 packed-FP16 convolution (reference: mat_mul.c:2189-2343) --
 * prm: iw, ih, ic, oc, batch, ow, oh, kw, kh, sx, sy, px, py, dx, dy, kp, np,
 * upscale (NativeConvParams order).  x: [batch][ic][ih][iw]; wperm: permuted
 * FP16 [kp][np]; out: [batch][oc][oh][ow].  im2col row pos = oy*ow + ox,
 * column col = ci*kh*kw + ky*kw + kx, then the opcode-16 GEMM in mode 3. */
void orc_conv2d_nchw_f16(float *out, const float *x, const uint16_t *wperm, const float *bias,
                         const int32_t *prm, int round_acc_f16);
/* One im2col matrix (FP32, [oh*ow][kp]) of batch b, as the reference gathers it. */
void orc_conv_im2col(float *a, const float *x, const int32_t *prm, int b);

/* ---- opcode 19 model auxiliaries (reference: mat_mul.c:2344-2480) --------
 * prm: mode, count, width, channels, spatial, groups, batch, other_count,
 * activation (NativeAuxParams order); eps.  w, b may be NULL where the mode
 * allows.  out holds `count` floats. */
void orc_model_aux(float *out, const float *x, const float *w, const float *b, const int32_t *prm, float eps);
/* x*sigmoid(z) activations of the epilogues: mode 1 GELU(tanh), 2 QuickGELU,
 * 4/5 SiLU (mat_mul.c:788-826). */
float orc_activation(float x, int mode);

/* ---- opcodes 2-4: ggml-block weights dequantised to FP16 -----------------
 * (reference: mat_mul.c:246-430 dequantisation, :1601-1874 GEMM; quants.h:11-31
 * block layouts).  The weight is a stream of K*N/256 super-blocks; super-block i
 * dequantises to FP16 elements [256i, 256i+256) of the packed FP16 weight
 * (orc_f16_perm_offset layout).  A super-block is 8 FP16 scales followed by the
 * codes (Q4_0 / IQ4_NL: 128 bytes of nibbles, Q8_0: 256 INT8); element e uses
 * scale e/32.  Q8_0: code = byte e.  Q4_0 / IQ4_NL: with v = e/64, i = e%64,
 * the nibble is the low (v < 2) or high (v >= 2) half of byte 2i + (v & 1);
 * value = nibble - 8 (Q4_0) or the IQ4_NL table entry.  The element is the
 * FP16 product code * scale rounded to nearest even (HVX qf16 multiply then
 * conversion; its ulp-level rounding is undocumented). */
#define ORC_GGML_Q4_0 2
#define ORC_GGML_Q8_0 8
#define ORC_GGML_IQ4_NL 20
/* Bytes of one 256-element super-block (144, 272), 0 for other types. */
size_t orc_qk0_block_bytes(int type);
/* FP16 bits of element e (0..255) of one super-block. */
uint16_t orc_qk0_element(const uint8_t *block, int type, int e);
/* Dequantised weight as FP16 bits, row-major w_nk[n][k]. */
void orc_qk0_dequant(uint16_t *w_nk, const uint8_t *src, int type, int k, int n);
/* Quantise FP32 w_kn[k][n] into the super-block stream (test data: the
 * inverse of orc_qk0_dequant up to the codec's rounding; scale per 32-element
 * group = the group's largest magnitude / 8, 127 or 127 for Q4_0, Q8_0,
 * IQ4_NL, codes by rounding to the nearest level). */
void orc_qk0_quantize(uint8_t *dst, const float *w_kn, int type, int k, int n);
/* out[i][c] = sum_k f16(x[row][k]) * W16(k, c) in FP32 (the reference reads
 * the accumulator through FP16, mat_mul.c:751-778: round_acc_f16 applies that
 * rounding); rows as in orc_f16_linear_rows. */
void orc_qk0_linear_rows(float *out, const float *x, const uint8_t *src, int type, int m, int k, int n,
                         int round_acc_f16, const int32_t *rows, int nrows);

/* Number of OpenMP threads this build uses (1 without OpenMP). */
int orc_threads(void);
/* Use n OpenMP threads from now on (ignored without OpenMP); launchers such as
   torchrun export OMP_NUM_THREADS=1, the CPU baseline wants every host thread. */
void orc_set_threads(int n);

#ifdef __cplusplus
}
#endif

#endif
