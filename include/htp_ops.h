/*
 * Host entry points of the reference's FastRPC interface (reference:
 * include/htp_ops.idl:9-27), implemented directly in libhtp_ops_b200.so.
 * There is no RPC hop: a handle names an in-process backend bound to a CUDA
 * device, and the calls run the B200 kernels.  Return values follow the
 * reference (AEE codes from the Hexagon SDK's AEEStdErr.h numbering, or the
 * negative operator codes of htp_ops_b200.h).
 */
#ifndef HTP_B200_HTP_OPS_H
#define HTP_B200_HTP_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uint64_t remote_handle64;
typedef int AEEResult;

/* AEEStdErr.h values used by the reference (commu.c) */
#ifndef AEE_SUCCESS
#define AEE_SUCCESS 0
#define AEE_EFAILED 1
#define AEE_ENOMEMORY 2
#define AEE_EBADSTATE 13
#define AEE_EBADPARM 14
#define AEE_EUNSUPPORTED 20
#define AEE_EALREADY 26
#endif

#define htp_ops_URI "file:///libhtp_ops_b200.so?htp_ops_skel_handle_invoke&_modver=1.0"

/* reference: commu.c:369-382 (open) and 385-409 (close) */
AEEResult htp_ops_open(const char *uri, remote_handle64 *handle);
AEEResult htp_ops_close(remote_handle64 handle);
/* reference: htp_ops.idl:10-16 / commu.c:412-587 */
AEEResult htp_ops_init_backend(remote_handle64 handle);
AEEResult htp_ops_init_backend_fraction(remote_handle64 handle, uint32_t numerator, uint32_t denominator);
AEEResult htp_ops_init_mapping_backend(remote_handle64 handle);
AEEResult htp_ops_release_backend(remote_handle64 handle);
AEEResult htp_ops_create_channel(remote_handle64 handle, int32_t fd, uint32_t size);
AEEResult htp_ops_create_channel_with_token(remote_handle64 handle, uint64_t session_token,
                                            int32_t fd, uint32_t size);
AEEResult htp_ops_destroy_channel(remote_handle64 handle);
/* reference: htp_ops.idl:19 — not part of this library's hot path: AEE_EUNSUPPORTED */
AEEResult htp_ops_rms_norm_f32(remote_handle64 handle, int32_t fd0, int32_t offset0, int32_t fd1,
                               int32_t offset1, int32_t ne0, int32_t ne1);
/* reference: htp_ops.idl:20-25 / commu.c:637-808 */
AEEResult htp_ops_mat_mul_permuted_w16a32(remote_handle64 handle, int32_t output_fd,
                                          int32_t output_offset, int32_t activation_fd,
                                          int32_t activation_offset, int32_t weight_fd,
                                          int32_t weight_offset, int32_t m, int32_t k, int32_t n);
AEEResult htp_ops_mat_mul_permuted_w16a32_trace(remote_handle64 handle, int32_t output_fd,
                                                int32_t output_offset, int32_t activation_fd,
                                                int32_t activation_offset, int32_t weight_fd,
                                                int32_t weight_offset, int32_t m, int32_t k, int32_t n,
                                                uint64_t *activation_hash, uint64_t *output_hash,
                                                uint64_t *output_hash_after_remap);
/* reference: htp_ops.idl:27 / commu.c:813-827 — runs this library's self-checks */
AEEResult htp_ops_test_ops(remote_handle64 handle, int32_t *userdma_scope);

#ifdef __cplusplus
}
#endif

#endif
