/*
 * Legacy op exports and capability markers (reference:
 * include/host/op_export.h:5-17, src/host/op_export.c:6-48).
 */
#ifndef HTP_B200_HOST_OP_EXPORT_H
#define HTP_B200_HOST_OP_EXPORT_H

#include <stdint.h>

#include "session.h"

#ifdef __cplusplus
extern "C" {
#endif

int htp_ops_rpc_rms_norm_f32(int dst_fd, int dst_offset, int src_fd, int src_offset, int ne0, int ne1);
int htp_ops_rpc_rms_norm_f32_session(htp_ops_session *session, int dst_fd, int dst_offset,
                                     int src_fd, int src_offset, int ne0, int ne1);
int htp_ops_rpc_mat_mul_permuted_w16a32(int output_fd, int output_offset, int activation_fd,
                                        int activation_offset, int weight_fd, int weight_offset,
                                        int m, int k, int n);
int htp_ops_rpc_mat_mul_permuted_w16a32_session(htp_ops_session *session, int output_fd,
                                                int output_offset, int activation_fd,
                                                int activation_offset, int weight_fd,
                                                int weight_offset, int m, int k, int n);
int htp_ops_rpc_mat_mul_permuted_w16a32_trace_session(htp_ops_session *session, int output_fd,
                                                      int output_offset, int activation_fd,
                                                      int activation_offset, int weight_fd,
                                                      int weight_offset, int m, int k, int n,
                                                      uint64_t *activation_hash, uint64_t *output_hash,
                                                      uint64_t *output_hash_after_remap);

/* Capability markers.  1 = the shared-message opcode-16 epilogue is served
 * (op_export.c:41).  The native-model / DiT auxiliary / DiT concat markers
 * return 0: those opcodes (17-19) are not executed by this library, which
 * tells callers to keep them on their own path. */
int htp_ops_f16_epilogue_version(void);
int htp_ops_native_model_version(void);
int htp_ops_dit_aux_version(void);
int htp_ops_dit_concat_version(void);
/* New marker (no reference counterpart): 1 = opcode 15 accepts the 56-byte
 * NativeW8A8EpilogueParams request (bias / GELU / QuickGELU / channel-major). */
int htp_ops_w8a8_epilogue_version(void);

#ifdef __cplusplus
}
#endif

#endif
