/*
 * Shim compiled against the READ-ONLY reference headers (include/message.h,
 * include/op_reg.h, include/dsp/f16_gemm_plan.h) into oracle/_ref/, and, with
 * -DSHIM_NO_PLANNER, against this repository's include/ headers.  It exposes
 * struct sizes/offsets and the message validator (and the reference's FP16
 * planner) so tests can diff this repository's wire ABI against the reference
 * compiled here.  TEST INFRASTRUCTURE ONLY.
 */
#include <stddef.h>
#include <stdint.h>

#include "message.h"
#include "op_reg.h"
#ifndef SHIM_NO_PLANNER
#include "dsp/f16_gemm_plan.h"
#endif

#define FIELD(s, f) offsetof(struct s, f)

/* name -> value table of layout facts; terminated by a NULL name */
struct ref_fact {
  const char *name;
  long value;
};

static const struct ref_fact facts[] = {
    {"sizeof.MessageState", sizeof(struct MessageState)},
    {"sizeof.MessageHeader", sizeof(struct MessageHeader)},
    {"sizeof.RequestHeader", sizeof(struct RequestHeader)},
    {"sizeof.OpComputeRequest", sizeof(struct OpComputeRequest)},
    {"sizeof.RpcmemMapRequest", sizeof(struct RpcmemMapRequest)},
    {"sizeof.RpcmemMapEntryV2", sizeof(struct RpcmemMapEntryV2)},
    {"sizeof.RpcmemMapRequestV2", sizeof(struct RpcmemMapRequestV2)},
    {"sizeof.RpcmemBufAddr", sizeof(struct RpcmemBufAddr)},
    {"sizeof.RmsNormF32Params", sizeof(struct RmsNormF32Params)},
    {"sizeof.W8A8Header", sizeof(struct W8A8Header)},
    {"sizeof.NativeW8A8Params", sizeof(struct NativeW8A8Params)},
    {"sizeof.NativeW8A8Profile", sizeof(struct NativeW8A8Profile)},
    {"sizeof.NativeW8A8ProfileParams", sizeof(struct NativeW8A8ProfileParams)},
    {"sizeof.W8A8CpuBatch", sizeof(struct W8A8CpuBatch)},
    {"sizeof.W8A8CpuControl", sizeof(struct W8A8CpuControl)},
    {"sizeof.NativeW8A8CpuParams", sizeof(struct NativeW8A8CpuParams)},
    {"sizeof.MatMulParams", sizeof(struct MatMulParams)},
    {"sizeof.F16EpilogueParams", sizeof(struct F16EpilogueParams)},
    {"offsetof.MessageHeader.checksum", FIELD(MessageHeader, checksum)},
    {"offsetof.MessageHeader.n_reqs", FIELD(MessageHeader, n_reqs)},
    {"offsetof.MessageHeader.req_offsets", FIELD(MessageHeader, req_offsets)},
    {"offsetof.RequestHeader.type", FIELD(RequestHeader, type)},
    {"offsetof.RequestHeader.data", FIELD(RequestHeader, data)},
    {"offsetof.RpcmemMapRequestV2.session_token", FIELD(RpcmemMapRequestV2, session_token)},
    {"offsetof.RpcmemMapRequestV2.entries", FIELD(RpcmemMapRequestV2, entries)},
    {"offsetof.W8A8Header.weight_offset", FIELD(W8A8Header, weight_offset)},
    {"offsetof.W8A8Header.bytes", FIELD(W8A8Header, bytes)},
    {"offsetof.W8A8Header.original_f16_signature", FIELD(W8A8Header, original_f16_signature)},
    {"offsetof.NativeW8A8Params.constants", FIELD(NativeW8A8Params, constants)},
    {"offsetof.NativeW8A8Params.m", FIELD(NativeW8A8Params, m)},
    {"offsetof.NativeW8A8Params.elapsed_us", FIELD(NativeW8A8Params, elapsed_us)},
    {"offsetof.NativeW8A8Profile.setup_ticks", FIELD(NativeW8A8Profile, setup_ticks)},
    {"offsetof.NativeW8A8Profile.readout_ticks", FIELD(NativeW8A8Profile, readout_ticks)},
    {"offsetof.W8A8CpuControl.weight_loaded_bytes", FIELD(W8A8CpuControl, weight_loaded_bytes)},
    {"offsetof.W8A8CpuControl.resident_batch_rows", FIELD(W8A8CpuControl, resident_batch_rows)},
    {"offsetof.W8A8CpuControl.scales", FIELD(W8A8CpuControl, scales)},
    {"offsetof.W8A8CpuControl.batches", FIELD(W8A8CpuControl, batches)},
    {"offsetof.NativeW8A8CpuParams.control", FIELD(NativeW8A8CpuParams, control)},
    {"offsetof.MatMulParams.m", FIELD(MatMulParams, m)},
    {"offsetof.MatMulParams.debug_vtcm_base", FIELD(MatMulParams, debug_vtcm_base)},
    {"offsetof.MatMulParams.debug_hmx_lock_result", FIELD(MatMulParams, debug_hmx_lock_result)},
    {"offsetof.MatMulParams.debug_dsp_output_hash_after_invalidate",
     FIELD(MatMulParams, debug_dsp_output_hash_after_invalidate)},
    {"offsetof.F16EpilogueParams.bias", FIELD(F16EpilogueParams, bias)},
    {"offsetof.F16EpilogueParams.m", FIELD(F16EpilogueParams, m)},
    {"offsetof.F16EpilogueParams.channels", FIELD(F16EpilogueParams, channels)},
    {"offsetof.F16EpilogueParams.mode", FIELD(F16EpilogueParams, mode)},
    {"offsetof.F16EpilogueParams.elapsed_us", FIELD(F16EpilogueParams, elapsed_us)},
    {"sizeof.NativeConvParams", sizeof(struct NativeConvParams)},
    {"offsetof.NativeConvParams.bias", FIELD(NativeConvParams, bias)},
    {"offsetof.NativeConvParams.iw", FIELD(NativeConvParams, iw)},
    {"offsetof.NativeConvParams.batch", FIELD(NativeConvParams, batch)},
    {"offsetof.NativeConvParams.kw", FIELD(NativeConvParams, kw)},
    {"offsetof.NativeConvParams.dy", FIELD(NativeConvParams, dy)},
    {"offsetof.NativeConvParams.kp", FIELD(NativeConvParams, kp)},
    {"offsetof.NativeConvParams.upscale", FIELD(NativeConvParams, upscale)},
    {"offsetof.NativeConvParams.elapsed_us", FIELD(NativeConvParams, elapsed_us)},
    {"offsetof.NativeConvParams.store_us", FIELD(NativeConvParams, store_us)},
    {"sizeof.NativeAuxParams", sizeof(struct NativeAuxParams)},
    {"offsetof.NativeAuxParams.mode", FIELD(NativeAuxParams, mode)},
    {"offsetof.NativeAuxParams.groups", FIELD(NativeAuxParams, groups)},
    {"offsetof.NativeAuxParams.activation", FIELD(NativeAuxParams, activation)},
    {"offsetof.NativeAuxParams.eps", FIELD(NativeAuxParams, eps)},
    {"offsetof.NativeAuxParams.elapsed_us", FIELD(NativeAuxParams, elapsed_us)},
    {"enum.HTP_OPS_RMS_NORM_F32", HTP_OPS_RMS_NORM_F32},
    {"enum.HTP_OPS_MAT_MUL_PERMUTED_W16A32", HTP_OPS_MAT_MUL_PERMUTED_W16A32},
    {"enum.HTP_OPS_MAT_MUL_NATIVE_W8A8", HTP_OPS_MAT_MUL_NATIVE_W8A8},
    {"enum.HTP_OPS_MAT_MUL_F16_EPILOGUE", HTP_OPS_MAT_MUL_F16_EPILOGUE},
    {"enum.HTP_OPS_CONV2D_NCHW_F16", HTP_OPS_CONV2D_NCHW_F16},
    {"enum.HTP_OPS_MODEL_AUX_F32", HTP_OPS_MODEL_AUX_F32},
    {"enum.HTP_OPS_COUNT", HTP_OPS_COUNT},
    {"enum.REQUEST_TYPE_OP_COMPUTE", REQUEST_TYPE_OP_COMPUTE},
    {"enum.REQUEST_TYPE_RPCMEM_MAP", REQUEST_TYPE_RPCMEM_MAP},
    {"enum.RPCMEM_MAP_REQUEST_SESSION_MAGIC", (long)RPCMEM_MAP_REQUEST_SESSION_MAGIC},
    {0, 0},
};

const struct ref_fact *ref_facts(void) { return facts; }

int ref_validate_layout(const void *msg, size_t capacity, size_t *total) {
  return message_header_validate_layout((const struct MessageHeader *)msg, capacity, total);
}

#ifndef SHIM_NO_PLANNER
int ref_f16_plan(int m, int k, int n, size_t vtcm, size_t reserved, size_t out[5]) {
  f16_gemm_plan_t p;
  if (!f16_gemm_make_plan(m, k, n, vtcm, reserved, &p)) return 0;
  out[0] = p.rows;
  out[1] = p.cols;
  out[2] = p.activation_bytes;
  out[3] = p.weight_bytes;
  out[4] = p.output_bytes;
  return 1;
}
#endif
