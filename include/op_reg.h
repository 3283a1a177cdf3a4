/*
 * Operator registry and packed request payloads for the linear-operator hot
 * path, byte-compatible with the reference library (reference:
 * include/op_reg.h:41-181, 477-489).
 *
 * Only the payloads of the ops this library executes are declared here:
 *   opcode  1  HTP_OPS_MAT_MUL_PERMUTED_W16A32  MatMulParams (92 B, 96 B with elapsed_us)
 *   opcodes 2-4 HTP_OPS_MAT_MUL_PERMUTED_W4D16A32, _W8D16A32, _W4D16A32_IQ4_NL
 *                                               MatMulParams; weight = ggml super-blocks
 *   opcode 15  HTP_OPS_MAT_MUL_NATIVE_W8A8      NativeW8A8Params (40 B), +profile (104 B),
 *                                               +CPU control (48 B), +epilogue (56 B, new)
 *   opcode 16  HTP_OPS_MAT_MUL_F16_EPILOGUE     F16EpilogueParams (56 B)
 *   opcode 17  HTP_OPS_CONV2D_NCHW_F16          NativeConvParams (124 B)
 *   opcode 19  HTP_OPS_MODEL_AUX_F32            NativeAuxParams (76 B)
 * The opcode numbering is the reference's, including the ops that are not
 * executed here (they are answered with AEE_EUNSUPPORTED by the dispatcher).
 */
#ifndef HTP_B200_OP_REG_H
#define HTP_B200_OP_REG_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum HtpOpsIndex {
  HTP_OPS_RMS_NORM_F32,                        /* 0 */
  HTP_OPS_MAT_MUL_PERMUTED_W16A32,             /* 1  (executed) */
  HTP_OPS_MAT_MUL_PERMUTED_W4D16A32,           /* 2  (executed) */
  HTP_OPS_MAT_MUL_PERMUTED_W8D16A32,           /* 3  (executed) */
  HTP_OPS_MAT_MUL_PERMUTED_W4D16A32_IQ4_NL,    /* 4  (executed) */
  HTP_OPS_FLASH_ATTN_QO_F32_KV_F16,            /* 5 */
  HTP_OPS_BLOCK_SPARSE_ATTN_QO_F32_KV_F16,     /* 6 */
  HTP_OPS_BLOCK_SPARSE_SCORE_QO_F32_KM_F16,    /* 7 */
  HTP_OPS_QKV_MUL_RMS_PACKED_W16A32,           /* 8 */
  HTP_OPS_BLOCK_SPARSE_ATTN_QKV_PACKED_F16,    /* 9 */
  HTP_OPS_QKV_MUL_RMS_PACKED_DUAL_W16A32,      /* 10 */
  HTP_OPS_QKV_MUL_RMS_PACKED_ROPE_W16A32,      /* 11 */
  HTP_OPS_QKV_MUL_RMS_PACKED_DUAL_ROPE_W16A32, /* 12 */
  HTP_OPS_FUSED_ANCHOR_ATTN_QO_F32_KV_F16,     /* 13 */
  HTP_OPS_ATTN_REARRANGE_BENCH,                /* 14 */
  HTP_OPS_MAT_MUL_NATIVE_W8A8,                 /* 15 (executed) */
  HTP_OPS_MAT_MUL_F16_EPILOGUE,                /* 16 (executed) */
  HTP_OPS_CONV2D_NCHW_F16,                     /* 17 */
  HTP_OPS_ATTENTION_F32,                       /* 18 */
  HTP_OPS_MODEL_AUX_F32,                       /* 19 */
  HTP_OPS_COUNT,
};

/* A tensor reference: a registered buffer (fd) plus a byte offset into it. */
struct RpcmemBufAddr {
  int32_t fd;
  int32_t offset;
} __attribute__((packed));

struct RmsNormF32Params {
  struct RpcmemBufAddr dst;
  struct RpcmemBufAddr src;
  int32_t ne0;
  int32_t ne1;
} __attribute__((packed));

/*
 * W8A8 constants blob, produced offline by the caller's packer.  Layout of the
 * blob (all offsets from the blob start):
 *   [0, 128)                   this header
 *   [weight_offset, +k*n)      INT8 weights in the HMX "deep" N64 layout
 *   [scale_offset, +4n)        FP32 per-column weight scale sw[n]
 *   [sum_offset, +4n)          INT32 column sums  sum_k w[n][k]
 *   [inverse_offset, +4k)      FP32 per-input-channel multiplier inverse[k]
 * magic = 0x38574d48 ("HMW8"), version = 1.
 */
struct W8A8Header {
  uint32_t magic, version, k, n;
  uint32_t weight_offset, scale_offset, sum_offset, inverse_offset, bytes, reserved;
  uint64_t original_f16_signature;
  uint8_t padding[80];
};

#define W8A8_HEADER_MAGIC 0x38574d48u
#define W8A8_HEADER_VERSION 1u

struct NativeW8A8Params {
  struct RpcmemBufAddr output, activation, constants;
  int32_t m, k, n, elapsed_us;
} __attribute__((packed));

/* Optional diagnostic trailer (104-byte request).  mode 1/2/3 as in the
 * reference; here the phase times are CUDA-event times in 19.2 MHz ticks so the
 * caller's tick arithmetic keeps working. */
struct NativeW8A8Profile {
  uint32_t mode, reserved;
  uint64_t setup_ticks, activation_ticks, weight_ticks, hmx_ticks, output_ticks;
  uint64_t mac_ticks, readout_ticks;
};
struct NativeW8A8ProfileParams {
  struct NativeW8A8Params base;
  struct NativeW8A8Profile profile;
} __attribute__((packed));

/* Opt-in "raw planes to the CPU" experiment (48-byte request). */
#define W8A8_CPU_MAX_BATCHES 64
#define W8A8_CONTROL_WEIGHT_FIRST 1u
struct W8A8CpuBatch {
  int32_t m0, rows, n0, columns;
};
struct W8A8CpuControl {
  uint32_t produced;
  uint32_t flags;
  uint32_t vtcm_bytes, activation_rows, weight_columns, weight_loads;
  uint64_t weight_loaded_bytes;
  uint32_t resident_batch_rows;
  uint8_t padding[92];
  float scales[4096];
  struct W8A8CpuBatch batches[W8A8_CPU_MAX_BATCHES];
};
struct NativeW8A8CpuParams {
  struct NativeW8A8Params base;
  struct RpcmemBufAddr control;
} __attribute__((packed));

/*
 * Extension (no reference counterpart): opcode 15 with the opcode-16 epilogue.
 * 56 bytes, distinct from the 40/48/104-byte opcode-15 requests, so an old
 * receiver rejects it (payload size check) instead of misreading it.
 * mode: 0 = bias, 1 = bias+GELU(tanh), 2 = bias+QuickGELU, 3 = bias + cropped
 * channel-major store out[c*m + row] for c < channels.  bias.fd < 0: no bias.
 */
struct NativeW8A8EpilogueParams {
  struct NativeW8A8Params base;
  struct RpcmemBufAddr bias;
  int32_t channels, mode;
} __attribute__((packed));

struct MatMulParams {
  struct RpcmemBufAddr output;
  struct RpcmemBufAddr activation; /* m * k FP32 */
  struct RpcmemBufAddr weight;     /* k * n FP16, permuted tile layout */
  int32_t m;
  int32_t k;
  int32_t n;
  /* Diagnostic fields; part of the wire layout even when tracing is off. */
  uint64_t debug_vtcm_base;
  uint32_t debug_vtcm_size;
  int32_t debug_vtcm_ctx;
  int32_t debug_hmx_ctx;
  uint64_t debug_worker_pool;
  int32_t debug_hmx_lock_result;
  uint64_t debug_dsp_activation_hash;
  uint64_t debug_dsp_output_hash;
  uint64_t debug_dsp_output_hash_after_invalidate;
} __attribute__((packed));

struct MatMulProfileParams {
  struct MatMulParams matmul;
  int32_t elapsed_us;
} __attribute__((packed));

/* mode: 0 = bias, 1 = bias+GELU, 2 = bias+QuickGELU, 3 = bias+NCHW store. */
struct F16EpilogueParams {
  struct RpcmemBufAddr output, activation, weight, bias;
  int32_t m, k, n, channels, mode, elapsed_us;
} __attribute__((packed));

/* Opcode 17: packed-FP16 2-D convolution, NCHW in and out (reference:
 * op_reg.h:491-495).  Input [batch][ic][ih][iw] FP32, optionally upsampled 2x
 * by nearest neighbour (upscale 2) before the convolution; weight: permuted
 * FP16 [kp][np] (the opcode-16 tile layout) with K index ci*kh*kw + ky*kw + kx
 * (kp >= ic*kh*kw, np >= oc, both multiples of 32); output [batch][oc][oh][ow]
 * FP32 = conv + bias.  The *_us fields are written back. */
struct NativeConvParams {
  struct RpcmemBufAddr output, activation, weight, bias;
  int32_t iw, ih, ic, oc, batch, ow, oh, kw, kh, sx, sy, px, py, dx, dy, kp, np, upscale;
  int32_t elapsed_us, gather_us, weight_us, hmx_us, store_us;
} __attribute__((packed));

/* Opcode 19: FP32 model auxiliaries around the linears (reference:
 * op_reg.h:503-508, mat_mul.c:2344-2480).  mode: 0 LayerNorm, 1 RMSNorm,
 * 2 GroupNorm, 3 broadcast add, 4 broadcast multiply, 5 SiLU, 6 GELU(tanh),
 * 7 QuickGELU, 8 [batch][width][spatial] -> [batch][spatial][width] transpose,
 * 9 LayerNorm + modulation (v + v*scale + shift), 10 gated residual
 * (x*gate + residual), 11 RoPE with 2x2 position matrices (into the attention
 * layout), 12 SwiGLU, 13 SwiGLU concatenated after an attention output.
 * activation: SiLU after the norms (modes 0-2, 9), or the gate/up order of
 * modes 12/13.  elapsed_us is written back. */
struct NativeAuxParams {
  struct RpcmemBufAddr output, input, weight, bias;
  int32_t mode, count, width, channels, spatial, groups, batch, other_count, activation;
  float eps;
  int32_t elapsed_us;
} __attribute__((packed));

#ifdef __cplusplus
#define HTPB_STATIC_ASSERT(c, msg) static_assert(c, msg)
#else
#define HTPB_STATIC_ASSERT(c, msg) _Static_assert(c, msg)
#endif

HTPB_STATIC_ASSERT(sizeof(struct W8A8Header) == 128, "W8A8 constants header ABI");
HTPB_STATIC_ASSERT(sizeof(struct NativeW8A8Params) == 40, "opcode 15 base payload ABI");
HTPB_STATIC_ASSERT(sizeof(struct NativeW8A8CpuParams) == 48, "opcode 15 CPU payload ABI");
HTPB_STATIC_ASSERT(sizeof(struct NativeW8A8EpilogueParams) == 56, "opcode 15 epilogue payload");
HTPB_STATIC_ASSERT(sizeof(struct W8A8CpuControl) == 17536, "W8A8 CPU control ABI");
HTPB_STATIC_ASSERT(offsetof(struct W8A8CpuControl, scales) == 128, "W8A8 control scales offset");
HTPB_STATIC_ASSERT(offsetof(struct W8A8CpuControl, batches) == 16512, "W8A8 control batches offset");
HTPB_STATIC_ASSERT(sizeof(struct NativeW8A8Profile) == 64, "W8A8 profile ABI");
HTPB_STATIC_ASSERT(sizeof(struct NativeW8A8ProfileParams) == 104, "opcode 15 profile payload ABI");
HTPB_STATIC_ASSERT(sizeof(struct MatMulParams) == 92, "opcode 1 payload ABI");
HTPB_STATIC_ASSERT(sizeof(struct MatMulProfileParams) == 96, "opcode 1 profile payload ABI");
HTPB_STATIC_ASSERT(sizeof(struct F16EpilogueParams) == 56, "opcode 16 payload ABI");
HTPB_STATIC_ASSERT(sizeof(struct NativeConvParams) == 124, "opcode 17 payload ABI");
HTPB_STATIC_ASSERT(sizeof(struct NativeAuxParams) == 76, "opcode 19 payload ABI");
HTPB_STATIC_ASSERT(HTP_OPS_MAT_MUL_PERMUTED_W16A32 == 1, "opcode 1");
HTPB_STATIC_ASSERT(HTP_OPS_MAT_MUL_NATIVE_W8A8 == 15, "opcode 15");
HTPB_STATIC_ASSERT(HTP_OPS_MAT_MUL_F16_EPILOGUE == 16, "opcode 16");

#ifdef __cplusplus
}
#endif

#endif /* HTP_B200_OP_REG_H */
