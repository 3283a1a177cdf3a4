/*
 * Session API of the host library (reference: include/host/session.h:15-49).
 * A session owns one backend handle (htp_ops.h) bound to the CUDA device that
 * is current when it is opened.  Reserved sessions get an index 1..31 used to
 * derive their channel token, as in the reference (session.c:52-57).
 */
#ifndef HTP_B200_HOST_SESSION_H
#define HTP_B200_HOST_SESSION_H

#include <stdint.h>

#include "../htp_ops.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct htp_ops_session htp_ops_session;

int htp_ops_session_open(htp_ops_session **out, int base_domain, const char *name, int reserve_new);
htp_ops_session *htp_ops_default_session(void);
int htp_ops_session_init_backend(htp_ops_session *session);
int htp_ops_session_acquire_backend(htp_ops_session *session);
int htp_ops_session_release_backend(htp_ops_session *session);
int htp_ops_session_create_channel(htp_ops_session *session, int fd, unsigned int max_msg_size);
int htp_ops_session_create_channel_with_token(htp_ops_session *session, int fd, unsigned int max_msg_size);
int htp_ops_session_destroy_channel(htp_ops_session *session);
remote_handle64 htp_ops_session_handle(const htp_ops_session *session);
int htp_ops_set_active_session(htp_ops_session *session);
int htp_ops_set_default_session(void);
uint32_t htp_ops_session_id(const htp_ops_session *session);
uint32_t htp_ops_session_domain(const htp_ops_session *session);
int htp_ops_session_is_reserved(const htp_ops_session *session);
int htp_ops_session_is_initialized(const htp_ops_session *session);
int htp_ops_session_has_channel(const htp_ops_session *session);
void htp_ops_session_close(htp_ops_session *session);

int open_dsp_session(int domain_id, int unsigned_pd_enabled);
void close_dsp_session(void);
remote_handle64 get_global_handle(void);
void init_htp_backend(void);
int release_htp_backend(void);
int create_htp_message_channel(int fd, unsigned int max_msg_size);
int destroy_htp_message_channel(void);

#ifdef __cplusplus
}
#endif

#endif
