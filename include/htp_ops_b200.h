/*
 * libhtp_ops_b200.so — C ABI of the B200 (sm_100a) linear-operator library.
 *
 * Two layers, both plain C (no torch types, plain pointers and sizes):
 *
 *  1. Device-pointer kernel API (htpg_* and the reference kernel names).
 *     Tensors live in HBM; work is enqueued on a CUDA stream (`stream` is a
 *     cudaStream_t passed as void*; NULL = the CUDA default stream).
 *     Calls return 0 or a negative error code and never synchronise unless
 *     stated.  These replace the DSP kernel entry points of the reference
 *     (include/dsp/ops.h:20-31).
 *
 *  2. The reference-facing host API (message channel, sessions, IDL names):
 *     declared in htp_ops.h, host/session.h and host/op_export.h of this
 *     include directory; it resolves {fd, offset} buffer references through the
 *     buffer registry below and calls layer 1.
 *
 * Error codes are the reference's (src/dsp/op_executor.cc:316-335,
 * src/dsp/ops/linear_w8a8.c:337-392, src/dsp/ops/mat_mul.c:939-955).
 */
#ifndef HTP_OPS_B200_H
#define HTP_OPS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- error codes ------------------------------------------------------ */
#define HTPG_OK 0
#define HTPG_EPAYLOAD (-1)   /* executor: bad payload size or shape */
#define HTPG_EUNMAPPED (-2)  /* executor: {fd,offset} not registered or too small */
#define HTPG_EHEADER (-3)    /* executor: constants header / alignment mismatch */
#define HTPG_EARGS (-10)     /* kernel: null pointer or shape out of range */
#define HTPG_ECAPACITY (-11) /* kernel: shape constraint (k%32, n%32/64, channels) */
#define HTPG_ECONTROL (-12)  /* kernel: alignment / control block */
#define HTPG_ELAUNCH (-13)   /* kernel: CUDA launch or stream error (worker submit in the reference) */
#define HTPG_ENOPLAN (-14)   /* kernel: no tile plan for this shape */
#define HTPG_EWATCHDOG (-16) /* device wait gave up (bounded spin expired); context stays usable */
#define HTPG_ENOMEM (-17)    /* device allocation failed */
#define HTPG_EARCH (-75)     /* device is not sm_100 */

/* Shape limits.  The reference admits M<=4096, K<=6144, N<=16384
 * (src/dsp/op_executor.cc:320); this build widens M and K (documented
 * extension) so the M=16384 and K=14336 configurations run. */
#define HTPG_W8A8_MAX_M 65536
#define HTPG_W8A8_MAX_K 16384
#define HTPG_W8A8_MAX_N 16384

/* Epilogue modes (include/op_reg.h F16EpilogueParams).  */
#define HTPG_MODE_BIAS 0
#define HTPG_MODE_GELU 1
#define HTPG_MODE_QUICK_GELU 2
#define HTPG_MODE_NCHW 3
/* Diagnostic mode of htpg_*_run / htpg_*_linear only (not on the wire): the
 * raw accumulators, row-major -- W8A8: the signed INT32 sum
 * sum_k (code-128)*w[n][k] (equal to the reference's acc - (colsum << 7)),
 * stored as int32; FP16: the FP32 accumulator. */
#define HTPG_MODE_RAW 4
/* W8A8 only: the reference's raw byte-plane export (the opcode-15 CPU-epilogue
 * layout).  For each 64-row tile (rows = its valid rows) and 32-column half,
 * byte p (LSB first) of the unsigned-code accumulator sum_k code_u8*w of
 * (m, n) is byte p*rows*32 + (m%64)*32 + n%32 of the half's stream, which
 * fills the half's 32 FP32 output columns of the tile's rows, 128 bytes a row.
 * The output must be dense (ldo = n). */
#define HTPG_MODE_PLANES 5

/* ---- library / device ------------------------------------------------- */
/* Select `device` for this thread and check it is sm_100.
 * Returns 0, HTPG_EARCH (not sm_100) or HTPG_ELAUNCH (no CUDA device). */
int htpg_init(int device);
/* Library version (1). */
int htpg_version(void);
/* Text for an error code. */
const char *htpg_strerror(int code);
/* Last CUDA error text recorded by the library on this thread ("" if none). */
const char *htpg_last_cuda_error(void);
/* Synchronise `stream`, then read and clear the device watchdog word.  Returns 0
 * when no device wait expired, HTPG_EWATCHDOG otherwise; *flags (optional)
 * receives the raw bits (bit 0: producer, 1: MMA, 2: epilogue wait expired). */
int htpg_check_device(void *stream, uint32_t *flags);

/* ---- activation quantisation (reference: linear_w8a8.c:34-128) --------- */
/* Per row m: x' = x*inverse[k]; scale = max(absmax(x')/127, 1e-12);
 * code = RNE(clamp(x'*(1/scale) + 128, 1, 255)) - 128 (int8, in [-127,127]).
 * inverse may be NULL (all ones).  codes: [m][k] int8; row_scales: [m]. */
int htpg_quantize_rows(int8_t *codes, float *row_scales, const float *x, const float *inverse,
                       int m, int k, void *stream);

/* ---- prepared weights ------------------------------------------------- */
typedef struct htpg_weights htpg_weights;
struct W8A8CpuControl; /* include/op_reg.h */
struct NativeW8A8Profile; /* include/op_reg.h */

/* Repack a W8A8 constants blob (device memory, reference layout:
 * include/op_reg.h W8A8Header) into the tensor-core layout; columns
 * [n0, n0+n_cols) only (n0, n_cols multiples of 64; n_cols = 0 means all).
 * Reads the 128-byte header once (synchronous).  Header errors: HTPG_EHEADER. */
int htpg_w8a8_weights_create(const void *constants, int k, int n, int n0, int n_cols,
                             void *stream, htpg_weights **out);
/* Repack a permuted FP16 weight (device memory, 32x32 tile layout of
 * src/host/test.c:552-556) into the tensor-core layout, columns [n0, n0+n_cols). */
int htpg_f16_weights_create(const uint16_t *permuted_weight, int k, int n, int n0, int n_cols,
                            void *stream, htpg_weights **out);
void htpg_weights_destroy(htpg_weights *w);
/* Columns held by a prepared weight. */
int htpg_weights_cols(const htpg_weights *w);

/* ---- linear operators on prepared weights ----------------------------- */
/* out = epilogue(dequant(quant(x) * W^T)) for the W8A8 path; see
 * htpg_w8a8_linear.  x: [m][k] FP32; out: [m][cols] (mode 0-2, row stride
 * ldo >= cols) or [channels][m] (mode 3, row stride ldo >= m); ldo = 0 means
 * dense.  bias: [cols] FP32 or NULL. */
int htpg_w8a8_run(const htpg_weights *w, float *out, int ldo, const float *x, const float *bias,
                  int m, int channels, int mode, void *stream);
int htpg_f16_run(const htpg_weights *w, float *out, int ldo, const float *x, const float *bias,
                 int m, int channels, int mode, void *stream);

/* Plane export on prepared weights: HTPG_MODE_PLANES into dst ([m][n] FP32
 * bytes), then fills `control` (host memory) as hmx_mat_mul_native_w8a8_cpu
 * does.  Synchronous.  No counterpart of this exact signature in the reference
 * (its kernel takes the constants blob). */
int htpg_w8a8_run_planes(const htpg_weights *w, float *dst, const float *x, int m,
                         struct W8A8CpuControl *control, void *stream);

/* ---- opcode 17: packed-FP16 2-D convolution, NCHW (reference:
 * mat_mul.c:2189-2343) ------------------------------------------------- */
/* On prepared FP16 weights (htpg_f16_weights_create(weight, kp, np, ...)):
 * per image, im2col (nearest 2x upsample when upscale = 2; FP16 round to
 * nearest) into an internal grow-only buffer, then the FP16 GEMM with the
 * bias + channel-major epilogue: dst [batch][oc][oh][ow].  Geometry checks as
 * the reference executor (HTPG_EPAYLOAD). */
struct NativeConvParams; /* include/op_reg.h */
int htpg_conv2d_run(const htpg_weights *w, float *dst, const float *x, const float *bias,
                    const struct NativeConvParams *p, void *stream);
/* Budget of the im2col staging buffer (default 256 MiB): each GEMM launch
 * covers max(128, bytes / (2*kp)) output rows of one image. */
int htpg_conv_set_chunk_bytes(size_t bytes);
/* The reference's kernel name: device pointers, the weight in the permuted FP16
 * layout [kp][np] (cached per pointer like the other one-call entry points);
 * synchronous; fills gather_us, weight_us, hmx_us, store_us. */
int hmx_conv2d_nchw_f16(float *dst, const float *input, const uint16_t *weight, const float *bias,
                        struct NativeConvParams *p);

/* ---- opcode 19: FP32 model auxiliaries (reference: mat_mul.c:2344-2480) -- */
/* All 14 modes of NativeAuxParams (include/op_reg.h) on device pointers; w and
 * b stand for the payload's weight/bias buffers (NULL = absent).  Checks as
 * the reference executor (HTPG_EPAYLOAD), plus GroupNorm's element count must
 * equal spatial*channels*batch. */
struct NativeAuxParams; /* include/op_reg.h */
int htpg_model_aux_check(const struct NativeAuxParams *p, int has_w, int has_b);
int htpg_model_aux(float *dst, const float *x, const float *w, const float *b,
                   const struct NativeAuxParams *p, void *stream);
/* The reference's kernel name; synchronous. */
int hvx_model_aux_f32(float *dst, const float *x, const float *w, const float *b,
                      const struct NativeAuxParams *p);

/* ---- opcodes 2-4: ggml-block weights (reference: mat_mul.c:246-430,
 *      1601-1874; quants.h:11-31; op_executor.cc:771-808) ------------------
 * The weight is the reference's permuted stream of K*N/256 super-blocks
 * (my_block_q4_0: 8 FP16 scales + 128 bytes of nibbles, 144 bytes;
 * my_block_q8_0: 8 FP16 scales + 256 INT8, 272 bytes), used in place (no
 * prepared copy).  weight_type is the ggml type: */
#define HTPG_GGML_Q4_0 2
#define HTPG_GGML_Q8_0 8
#define HTPG_GGML_IQ4_NL 20
/* Bytes of the super-block stream (0 for an unsupported type or shape). */
size_t htpg_qk0_weight_bytes(int weight_type, int k, int n);
/* Prepared weight (destroy with htpg_weights_destroy): the super-blocks
 * reordered once into per-stage records (128 columns x 64 k each, zero-padded
 * past N and K), so that the fused kernel loads a stage with one copy.  The
 * caller's buffer is not used afterwards. */
int htpg_qk0_weights_create(const void *weight, int k, int n, int weight_type, void *stream, htpg_weights **out);
/* out[m][n] = fp16(x[m][k]) * dequant(W) on a prepared weight (see below). */
int htpg_qk0_run(const htpg_weights *w, float *out, const float *x, int m, void *stream);
/* out[m][n] (FP32) = fp16(x[m][k]) * W16, FP32 accumulation.  M <= 32: one
 * fused kernel that dequantises weight tiles on the fly; larger M: the weight
 * is dequantised to FP16 in a stream-private scratch buffer and the FP16 GEMM
 * runs on it.  Device pointers, x and weight 16-byte aligned.  The prepared
 * weight is cached by address like the other one-call entry points. */
int htpg_qk0_linear(float *out, const float *x, const void *weight, int m, int k, int n, int weight_type,
                    void *stream);
/* The dequantised weight as FP16 bits, row-major w_nk[n][k]. */
int htpg_qk0_dequantize(uint16_t *w_nk, const void *weight, int k, int n, int weight_type, void *stream);
/* Plan of the fused kernel: {bn, tiles_a, tiles_b, k-blocks, CTAs, shared bytes}. */
int htpg_qk0_plan_info(int weight_type, int m, int n, int k, int sms, int64_t out[6]);
/* Plan of the register-fed decode kernel (m <= 32): {CTAs per SM, weight tiles
 * per CTA, 32-column tiles, 32-deep k-tiles, k ranges, CTAs, activation slice
 * bytes, shared bytes per CTA}.  HTPG_ENOPLAN when a shape forced with
 * htpg_set_qdec_shape does not fit. */
int htpg_qk0_decode_plan_info(int weight_type, int m, int n, int k, int sms, int64_t out[8]);

/* ---- column-sharded run with a fused output exchange -------------------- */
/* Multi-GPU form of htpg_w8a8_run for a weight split by output columns (N)
 * across ranks, each rank holding a column block: the epilogue stores every
 * finished output tile to each of outs[0..n_outs) (n_outs <= 8) with TMA, so
 * one launch both computes this rank's column block
 * and writes it into every rank's row-major [M][N] output over NVLink.  outs[i]
 * points at the block's first column in buffer i (its row pitch is ldo floats,
 * ldo = the full N); peers' buffers come from htpg_ipc_import.  Needs the
 * TMA-store epilogue: mode 0-2, 16-byte aligned blocks, M > 32 (else
 * HTPG_ECAPACITY).  The stores to peers are complete when the launch is; the
 * caller orders the ranks after it (e.g. a stream-ordered all-reduce of a token)
 * before anyone reads the assembled output.  No counterpart in the reference
 * (it has no multi-device path). */
int htpg_w8a8_run_gather(const htpg_weights *w, float *const *outs, int n_outs, int ldo, const float *x,
                         const float *bias, int m, int channels, int mode, void *stream);
/* CUDA IPC for peer buffers: export a device address as a 72-byte handle
 * (cudaIpcMemHandle_t of its allocation + the byte offset into it), import a
 * peer's handle as a local address (peer access enabled lazily), close it. */
#define HTPG_IPC_HANDLE_BYTES 72
int htpg_ipc_export(const void *dev_ptr, void *handle);
int htpg_ipc_import(const void *handle, void **dev_ptr);
int htpg_ipc_close(void *dev_ptr);

/* ---- W8A8 run that allocates nothing (no counterpart in the reference) -- */
/* For callers that must not allocate device memory per call: code running
 * under a fixed memory budget or a caching allocator that owns all device
 * memory, real-time loops where cudaMalloc's implicit device synchronisation
 * is not acceptable, and hosts that prepare every buffer up front.  Same
 * arguments, checks and results as htpg_w8a8_run for modes 0-4 (mode 5, the
 * plane export, is refused with HTPG_ECAPACITY), but the activation codes,
 * row scales and split-K partial sums live in one fixed static device array
 * of HTPG_STATIC_SCRATCH_BYTES per device instead of the per-stream
 * workspace, and no call allocates: no cudaMalloc, cudaFree or allocating
 * library routine.  Layout of the array: the split-K area (2,101,248 bytes,
 * cleared by every call that uses it), then m*k bytes of codes, then 4*m
 * bytes of row scales, each rounded up to 1 KiB; a call that needs more than
 * HTPG_STATIC_SCRATCH_BYTES returns HTPG_ESCRATCH and launches nothing
 * (m*k up to 31,453,184 - 4*m: e.g. M = 16384 at K = 1536).  The prepared
 * weight `w` is made beforehand with htpg_w8a8_weights_create, which does
 * allocate.  The first call on each device does that device's one-time set-up
 * (device properties and the array's device address), so make it before any
 * stream capture; each tile plan's kernel also sets its launch attributes on
 * its first use, and under CUDA's lazy module loading (the default) loads its
 * module then, so run each shape once before a capture.  Every call on a device shares the one array,
 * which keeps the previous call's contents: calls whose executions overlap on
 * the GPU (different streams, or host threads racing on one device) race on
 * it; order them on one stream. */
#define HTPG_STATIC_SCRATCH_BYTES (32u << 20)
#define HTPG_ESCRATCH (-18) /* request does not fit HTPG_STATIC_SCRATCH_BYTES */
int htpg_w8a8_run_static(const htpg_weights *w, float *out, int ldo, const float *x,
                         const float *bias, int m, int channels, int mode, void *stream);

/* ---- one-call linear operators (weights cached by pointer) ------------- */
/* W8A8 linear, opcode 15 (reference: linear_w8a8.c:327-530) plus the
 * optional opcode-16 epilogue (extension).  constants: device copy of the
 * blob.  The repacked weight is cached keyed by (address, k, n): a caller that
 * rewrites a blob in place, or frees it and may get the same address for a
 * different weight (caching allocators do), calls
 * htpg_weight_cache_drop(address) first.  The same holds for every one-call
 * entry point below (hmx_* names, htpg_f16_linear, hmx_conv2d_nchw_f16). */
int htpg_w8a8_linear(float *out, const float *x, const void *constants, const float *bias,
                     int m, int k, int n, int channels, int mode, void *stream);
/* Packed FP16 GEMM with fused epilogue, opcodes 1 and 16
 * (reference: mat_mul.c:937-1049).  FP32 accumulate. */
int htpg_f16_linear(float *out, const float *x, const uint16_t *permuted_weight, const float *bias,
                    int m, int k, int n, int channels, int mode, void *stream);
void htpg_weight_cache_drop(const void *weights);
void htpg_weight_cache_clear(void);

/* Per-phase device times (ms) of the last htpg_*_linear / run call on this
 * thread when profiling is on (htpg_set_profiling(1)); used for the opcode-15
 * profile trailer. */
int htpg_set_profiling(int on);
int htpg_last_phase_ms(float *quant_ms, float *gemm_ms, float *total_ms);
/* Fill the opcode-15 profile trailer (include/op_reg.h NativeW8A8Profile;
 * reference op_reg.h:91-101, linear_w8a8.c:328-335, 396-399, 421-508) for an
 * m x k x n run that just finished with profiling on: profile->mode (1, 2 or 3)
 * is kept, every other field rewritten.  setup_ticks = setup_ms, and
 * activation_ticks / hmx_ticks = this thread's last phase times, all in
 * 19.2 MHz ticks; weight_ticks and output_ticks stay 0 (the weight stream and
 * the output stores run inside the GEMM launch); mode 2: mac_ticks =
 * hmx_ticks; mode 3: reserved = 64-row activation tiles | 64-column weight
 * groups << 16 of one output tile (bit 31, the reference's table hit, stays 0),
 * mac_ticks = weight tiles loaded, readout_ticks = weight bytes loaded.  Used
 * by both hmx_mat_mul_native_w8a8_profiled and the 104-byte executor request. */
int htpg_w8a8_profile_fill(int m, int k, int n, double setup_ms, struct NativeW8A8Profile *profile);

/* Phase timing for benchmarks: while on, every run records CUDA events on its
 * stream before the activation pass, between it and the GEMM, and after the
 * GEMM, without synchronising.  htpg_phase_timing_read synchronises those
 * events, returns the summed device milliseconds of both phases and the
 * number of runs since the last read, and resets the sums. */
int htpg_phase_timing(int on);
int htpg_phase_timing_read(double *act_ms, double *gemm_ms, int *runs);

/* Kernel launches issued by this library since load (for launch accounting). */
uint64_t htpg_launch_count(void);

/* Diagnostic (no counterpart in the reference): one kernel that reads `bytes`
 * of device memory at `src` (a multiple of 32 bytes, 32-byte aligned) with the
 * decode kernels' 32-byte streaming loads and discards the data: the HBM read
 * ceiling that the weight-streaming decode kernels are measured against. */
int htpg_stream_read(const void *src, size_t bytes, void *stream);

/* Test hooks (no counterpart in the reference).  htpg_debug_simulate_abort
 * leaves, on the current device, the state a launch that gave up can leave:
 * every stream workspace (W8A8/FP16 split-K areas, opcode 2-4 stream-K
 * scratch) filled with the byte `fill` and the watchdog word set.  The next
 * htpg_check_device must then answer HTPG_EWATCHDOG and restore the zeroed
 * scratch that later launches rely on.  htpg_debug_workspaces reports the
 * bytes held by the stream workspaces of the current device. */
int htpg_debug_simulate_abort(uint32_t fill);
int htpg_debug_workspaces(size_t *ws_bytes, size_t *qws_bytes);

/* Tile plan the library uses for an m x n x k problem (kind 0 = W8A8,
 * 1 = FP16) with a row-major output on a device with `sms` SMs.  out[0..11] =
 * swap, bn, splits, tiles_a, tiles_b, kb_total, kb_per_split, units, grid,
 * smem bytes, full_units, tail_s.  swap = 0: activation rows are the MMA M
 * (128-row tiles, or 256-row CTA-pair tiles when tiles_a = ceil(m/256)), bn
 * weight columns per tile; 1: small-M swapped tiles (weights are the MMA M);
 * 2: the register-fed decode kernel (W8A8, m <= 16), bn = 8 or 16 activation
 * rows, tiles_a = 16-column groups, units = work chunks; 3: CTA-pair tiles in
 * the swapped orientation, tiles_a = 256-column weight tiles, bn activation
 * rows per tile, stores straight from registers.  For swap = 3, tail_s > 1
 * means the tiles after the first full_units (a last round of tiles that would
 * leave at least half of the SM pairs idle) are each cut into tail_s pieces of
 * consecutive k-blocks, one piece per pair, which exchange their exact INT32
 * sums so that each finishes a share of the tile's rows: units = full_units
 * + tail tiles x tail_s.
 * Otherwise full_units = units and tail_s = 1. */
int htpg_plan_info(int kind, int m, int n, int k, int sms, int64_t out[12]);

/* W8A8 CTA-pair plans with a row-major output of one destination (modes 0-2
 * and 4): 1 (default) run them in the swapped orientation, whose epilogue
 * writes each output row's 32 columns from registers as one 128-byte line;
 * 0 keep the normal orientation, whose epilogue stages 32 x 32 tiles in shared
 * memory for TMA stores.  Both give identical results; the switch exists for
 * measurement. */
int htpg_set_pair_direct(int on);

/* Swapped CTA-pair plans whose last round of tiles would leave at least half
 * of the SM pairs idle: 1 (default) cut those tiles into K pieces (see
 * htpg_plan_info), 0 keep whole tiles.  Results are identical (the pieces'
 * INT32 sums are exact); the switch exists for measurement and tests. */
int htpg_set_pair_tail_split(int on);

/* Which kernel runs opcode 2-4 (ggml-block weight) problems with m <= 32:
 * 0 (default) the register-fed decode kernel (each warp streams a 32-column
 * weight tile's super-blocks through a shared-memory ring into registers and
 * feeds mma.sync; k ranges summed in a fixed order) where it is the faster
 * one, else the tcgen05 kernel; 1 always the tcgen05 kernel; 2 always the
 * register-fed kernel.  Both are deterministic and
 * within 1e-5 (relative) of the FP32-accumulating oracle; they sum in
 * different orders. */
int htpg_set_qk0_decode(int which);

/* The register-fed opcode 2-4 decode kernel's launch shape: per_sm CTAs per
 * SM (1 or 2) with `tiles` 32-column weight tiles each (16, 8 or 4; narrower
 * CTAs put 2 or 4 warps on each tile).  (0, 0), the default, lets the planner
 * choose.  A forced shape that does not fit the problem makes the call return
 * HTPG_ENOPLAN.  Results do not depend on the shape beyond the order of the
 * k-range sums (each shape is deterministic); the switch exists for tests and
 * measurement. */
int htpg_set_qdec_shape(int per_sm, int tiles);

/* Which kernel runs W8A8 problems with m <= 16: 0 (default) the register-fed
 * decode kernel, 1 the swapped tcgen05 kernel that also serves 16 < m <= 32.
 * Both give identical results; the switch exists for measurement. */
int htpg_set_decode_kernel(int which);


/* ---- reference kernel-level names (reference: include/dsp/ops.h:20-31) ---
 * Same arguments and return codes as the DSP kernels, on device pointers;
 * synchronous (they return once the output is written).  The FP16 weight
 * type __fp16 of the reference is passed as its 16-bit pattern. */
int hmx_mat_mul_native_w8a8(float *dst, const float *activation, const uint8_t *constants, int m,
                            int k, int n);
int hmx_mat_mul_native_w8a8_profiled(float *dst, const float *activation, const uint8_t *constants,
                                     int m, int k, int n, struct NativeW8A8Profile *profile);
/* CPU-epilogue form of opcode 15 (reference: linear_w8a8.c:205-227, 512-526):
 * dst receives the raw byte planes of the unsigned-code INT32 accumulators
 * (see HTPG_MODE_PLANES) instead of FP32 values, and the control block (host
 * memory, include/op_reg.h W8A8CpuControl) the row scales, one batch
 * {0, m, 0, n/64} and produced = 1 (published last).  m <= 4096 (the control
 * block holds 4096 row scales); -12 when control is NULL. */
int hmx_mat_mul_native_w8a8_cpu(float *dst, const float *activation, const uint8_t *constants,
                                int m, int k, int n, struct W8A8CpuControl *control);
int hmx_mat_mul_f16_epilogue(float *dst, const float *activation, const uint16_t *weight,
                             const float *bias, int m, int k, int n, int channels, int mode);
int hmx_mat_mul_permuted_w16a32(float *dst, const float *activation,
                                const uint16_t *permuted_weight, int m, int k, int n);
/* opcodes 2-4 (include/dsp/ops.h:60 of the reference): returns 0 or -1. */
int hmx_mat_mul_permuted_qk_0_d16a32(float *dst, const float *activation, const uint8_t *permuted_weight,
                                     int m, int k, int n, int weight_type);

/* ---- buffer registry (replaces the DSP fd->pointer map cache,
 *      src/dsp/mmap_mgr.cc:10-139) ----------------------------------------- */
#define HTPG_BUF_DEVICE 0 /* HBM; ops read/write it directly */
#define HTPG_BUF_HOST 1   /* pinned host memory; ops stage through HBM */

/* Allocate a buffer of `bytes` (kind DEVICE: cudaMalloc; HOST: pinned host)
 * and register it; *fd receives a new descriptor, *ptr the address. */
int htpg_buffer_alloc(size_t bytes, int kind, int *fd, void **ptr);
/* Register caller-owned memory under a caller-chosen fd (>= 0). */
int htpg_buffer_register(int fd, void *ptr, size_t bytes, int kind);
/* Forget fd (frees it if the library allocated it); drops cached repacks. */
int htpg_buffer_release(int fd);
/* Mark fd's contents as rewritten: cached weight repacks taken from it are dropped. */
int htpg_buffer_touch(int fd);
/* Resolve {fd, offset} with `size` bytes needed; NULL if unknown / too small. */
void *htpg_buffer_resolve(int fd, int64_t offset, size_t size, int *kind);

/* Execute one OpComputeRequest (reference: src/dsp/op_executor.cc:274).
 * `req` points at the OpComputeRequest; req_size includes its payload.
 * Synchronous: returns after the device work finished (output visible to
 * host-kind buffers).  Returns the RequestHeader.state value. */
struct OpComputeRequest;
int execute_op_simple(struct OpComputeRequest *req, size_t req_size);

#ifdef __cplusplus
}
#endif

#endif /* HTP_OPS_B200_H */
