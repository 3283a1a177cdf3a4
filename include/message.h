/*
 * Shared-memory message channel framing, byte-compatible with the reference
 * library's wire format (reference: include/message.h:6-129).
 *
 * A channel is one caller-owned buffer.  The caller writes a MessageHeader,
 * n_reqs+1 request offsets and the requests, then sets state.v[0] = 1.  The
 * receiver (here: a host thread of libhtp_ops_b200.so that launches CUDA work)
 * runs every request, writes each RequestHeader.state, and sets state.v[1] = 1.
 *
 * The struct layouts, field names and the validator's accept/reject rules are
 * kept identical on purpose: existing callers (the sd.cpp HTP backend) build
 * these bytes themselves and must not notice the change of device.
 */
#ifndef HTP_B200_MESSAGE_H
#define HTP_B200_MESSAGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* 8 status bytes; v[0] = "request posted", v[1] = "request done". */
struct MessageState {
  union {
    volatile uint8_t v[8];
    volatile uint64_t d;
  };
} __attribute__((packed));

struct MessageHeader {
  struct MessageState state;
  uint32_t checksum;
  int32_t n_reqs;
  int32_t req_offsets[0]; /* n_reqs + 1 byte offsets from the header start */
} __attribute__((packed));

struct RequestHeader {
  int32_t state; /* written by the receiver: 0 or a negative error code */
  int32_t type;  /* enum RequestType */
  uint8_t data[0];
} __attribute__((packed));

enum RequestType {
  REQUEST_TYPE_NO_OP = 0,
  REQUEST_TYPE_RPCMEM_MAP,
  REQUEST_TYPE_OP_COMPUTE,
  REQUEST_TYPE_COUNT,
};

struct RpcmemMapRequest {
  int32_t n_puts;
  int32_t n_gets;
  int32_t fds[0];
} __attribute__((packed));

enum {
  RPCMEM_MAP_REQUEST_VERSION_LEGACY = 1,
  RPCMEM_MAP_REQUEST_VERSION_SESSION = 2,
  RPCMEM_MAP_REQUEST_SESSION_MAGIC = 0x32504d52u, /* "RMP2" */
};

struct RpcmemMapEntryV2 {
  int32_t fd;
  uint32_t role;
  uint64_t offset;
  uint64_t size;
  uint64_t producer_epoch;
} __attribute__((packed));

struct RpcmemMapRequestV2 {
  uint32_t magic;
  uint16_t version;
  uint16_t header_size;
  uint64_t session_token;
  int32_t n_puts;
  int32_t n_gets;
  struct RpcmemMapEntryV2 entries[0];
} __attribute__((packed));

struct OpComputeRequest {
  uint32_t op; /* enum HtpOpsIndex */
  uint8_t payload[0];
} __attribute__((packed));

/*
 * Returns 1 when the header, its offset table and every request span lie
 * inside `capacity` bytes, offsets are non-decreasing and every request holds
 * at least a RequestHeader; *total_size then receives the end of the last
 * request.  Returns 0 otherwise.  Same rules as the reference validator
 * (include/message.h:68-113).
 */
static inline int message_header_validate_layout(const struct MessageHeader *h, size_t capacity,
                                                 size_t *total_size) {
  const size_t fixed = sizeof(struct MessageHeader);
  if (!h || !total_size || capacity < fixed + sizeof(int32_t)) return 0;
  if (h->n_reqs < 0) return 0;
  const size_t n_offsets = (size_t)h->n_reqs + 1;
  if (n_offsets > (capacity - fixed) / sizeof(int32_t)) return 0;
  const size_t table_end = fixed + n_offsets * sizeof(int32_t);
  if (h->req_offsets[0] < 0) return 0;
  size_t cursor = (size_t)h->req_offsets[0];
  if (cursor < table_end || cursor > capacity) return 0;
  for (int32_t i = 1; i <= h->n_reqs; ++i) {
    if (h->req_offsets[i] < 0) return 0;
    const size_t next = (size_t)h->req_offsets[i];
    if (next < cursor || next > capacity || next - cursor < sizeof(struct RequestHeader)) return 0;
    cursor = next;
  }
  *total_size = cursor;
  return 1;
}

static inline size_t message_header_size(const struct MessageHeader *h) {
  return sizeof(struct MessageHeader) + ((size_t)h->n_reqs + 1) * sizeof(int32_t);
}

static inline size_t message_total_size(const struct MessageHeader *h) {
  return (size_t)h->req_offsets[h->n_reqs];
}

static inline size_t message_header_get_request_size(const struct MessageHeader *h, int req_idx) {
  return (size_t)(h->req_offsets[req_idx + 1] - h->req_offsets[req_idx]);
}

static inline struct RequestHeader *message_header_get_request_ptr(struct MessageHeader *h,
                                                                   int req_idx) {
  return (struct RequestHeader *)((uint8_t *)h + h->req_offsets[req_idx]);
}

#ifdef __cplusplus
}
#endif

#endif /* HTP_B200_MESSAGE_H */
