// Host runtime of libhtp_ops_b200.so: the reference's DSP-side plumbing
// rebuilt for a CUDA device.
//
//  * buffer registry      fd -> {pointer, size, kind}      (src/dsp/mmap_mgr.cc)
//  * execute_op_simple    payload validation, {fd,offset} resolution, host
//                         staging, kernel call, elapsed_us (src/dsp/op_executor.cc:274-540)
//  * message channel      receiver thread running the state.v[0] / v[1]
//                         protocol over a caller-owned host buffer (src/dsp/commu.c:99-347)
//  * backends / sessions  the FastRPC IDL names, session leases, legacy
//                         wrappers and capability markers (commu.c:369-827,
//                         src/host/session.c, src/host/op_export.c)
//
// "Cache invalidate" of an input becomes a host->device copy when the buffer
// is host memory, and "flush" of an output a device->host copy; device-memory
// buffers are used in place.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <climits>
#include <set>
#include <thread>
#include <tuple>
#include <vector>

#include "../../../include/host/op_export.h"
#include "../../../include/host/session.h"
#include "../../../include/htp_ops.h"
#include "../../../include/htp_ops_b200.h"
#include "../../../include/message.h"
#include "../../../include/op_reg.h"

namespace {

// ================================================================ registry
struct Buffer {
  void *ptr = nullptr;
  size_t bytes = 0;
  int kind = HTPG_BUF_DEVICE;
  bool owned = false;
  uint64_t generation = 0;
};

std::recursive_mutex g_reg_mu;
std::map<int, Buffer> g_buffers;
int g_next_fd = 1 << 20;  // library-chosen descriptors stay clear of small caller fds

// prepared weights of the executor, keyed by (fd, offset, generation, kind, k, n)
typedef std::tuple<int, int64_t, uint64_t, int, int, int> WeightKey;
std::map<WeightKey, htpg_weights *> g_exec_weights;

void drop_fd_weights(int fd) {
  for (auto it = g_exec_weights.begin(); it != g_exec_weights.end();) {
    if (std::get<0>(it->first) == fd) {
      htpg_weights_destroy(it->second);
      it = g_exec_weights.erase(it);
    } else {
      ++it;
    }
  }
}

bool lookup(int fd, int64_t offset, size_t size, Buffer *out) {
  std::lock_guard<std::recursive_mutex> lk(g_reg_mu);
  auto it = g_buffers.find(fd);
  if (it == g_buffers.end() || offset < 0) return false;
  const Buffer &b = it->second;
  if (static_cast<size_t>(offset) > b.bytes || size > b.bytes - static_cast<size_t>(offset)) return false;
  *out = b;
  return true;
}

}  // namespace

extern "C" int htpg_buffer_alloc(size_t bytes, int kind, int *fd, void **ptr) {
  if (!fd || !ptr || bytes == 0 || (kind != HTPG_BUF_DEVICE && kind != HTPG_BUF_HOST)) return HTPG_EARGS;
  void *p = nullptr;
  const cudaError_t e = kind == HTPG_BUF_DEVICE ? cudaMalloc(&p, bytes) : cudaMallocHost(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return HTPG_ENOMEM;
  }
  std::lock_guard<std::recursive_mutex> lk(g_reg_mu);
  while (g_buffers.count(g_next_fd)) ++g_next_fd;
  const int f = g_next_fd++;
  Buffer b;
  b.ptr = p;
  b.bytes = bytes;
  b.kind = kind;
  b.owned = true;
  g_buffers[f] = b;
  *fd = f;
  *ptr = p;
  return HTPG_OK;
}

extern "C" int htpg_buffer_register(int fd, void *ptr, size_t bytes, int kind) {
  if (fd < 0 || !ptr || bytes == 0 || (kind != HTPG_BUF_DEVICE && kind != HTPG_BUF_HOST)) return HTPG_EARGS;
  std::lock_guard<std::recursive_mutex> lk(g_reg_mu);
  auto it = g_buffers.find(fd);
  if (it != g_buffers.end()) {
    if (it->second.owned) return HTPG_EARGS;  // library-owned descriptors are not re-bound
    drop_fd_weights(fd);
  }
  Buffer b;
  b.ptr = ptr;
  b.bytes = bytes;
  b.kind = kind;
  b.generation = it != g_buffers.end() ? it->second.generation + 1 : 0;
  g_buffers[fd] = b;
  return HTPG_OK;
}

extern "C" int htpg_buffer_release(int fd) {
  std::lock_guard<std::recursive_mutex> lk(g_reg_mu);
  auto it = g_buffers.find(fd);
  if (it == g_buffers.end()) return HTPG_EUNMAPPED;
  drop_fd_weights(fd);
  if (it->second.owned) {
    if (it->second.kind == HTPG_BUF_DEVICE)
      cudaFree(it->second.ptr);
    else
      cudaFreeHost(it->second.ptr);
  }
  g_buffers.erase(it);
  return HTPG_OK;
}

extern "C" int htpg_buffer_touch(int fd) {
  std::lock_guard<std::recursive_mutex> lk(g_reg_mu);
  auto it = g_buffers.find(fd);
  if (it == g_buffers.end()) return HTPG_EUNMAPPED;
  drop_fd_weights(fd);
  ++it->second.generation;
  return HTPG_OK;
}

extern "C" void *htpg_buffer_resolve(int fd, int64_t offset, size_t size, int *kind) {
  Buffer b;
  if (!lookup(fd, offset, size, &b)) return nullptr;
  if (kind) *kind = b.kind;
  return static_cast<uint8_t *>(b.ptr) + offset;
}

// ================================================================ executor
namespace {

// A tensor operand of one request, resolved and (for host buffers) staged.
struct Operand {
  bool present = false;
  int fd = -1;
  int64_t offset = 0;
  size_t bytes = 0;
  Buffer buf;
  void *host = nullptr;    // caller-visible address
  void *device = nullptr;  // address the kernels use
};

// Device staging arena for host-memory operands (grow-only).
struct Staging {
  void *base = nullptr;
  size_t bytes = 0;
};
std::mutex g_exec_mu;  // requests execute one at a time, like the DSP receiver
Staging g_staging;

int resolve(Operand &o, int fd, int32_t offset, size_t bytes) {
  o.fd = fd;
  o.offset = offset;
  o.bytes = bytes;
  if (!lookup(fd, offset, bytes, &o.buf)) return -1;
  o.present = true;
  o.host = static_cast<uint8_t *>(o.buf.ptr) + offset;
  o.device = o.buf.kind == HTPG_BUF_DEVICE ? o.host : nullptr;
  return 0;
}

// Give every host-kind operand a device copy region; copy inputs in.
int stage_in(std::vector<Operand *> inputs, std::vector<Operand *> outputs) {
  size_t need = 0;
  auto add = [&](Operand *o) {
    if (o && o->present && o->buf.kind == HTPG_BUF_HOST) need += (o->bytes + 255) / 256 * 256;
  };
  for (auto *o : inputs) add(o);
  for (auto *o : outputs) add(o);
  if (need > g_staging.bytes) {
    if (g_staging.base) {
      cudaDeviceSynchronize();
      cudaFree(g_staging.base);
    }
    g_staging.base = nullptr;
    g_staging.bytes = 0;
    if (cudaMalloc(&g_staging.base, need) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ENOMEM;
    }
    g_staging.bytes = need;
  }
  size_t off = 0;
  auto place = [&](Operand *o, bool copy_in) -> int {
    if (!o || !o->present || o->buf.kind != HTPG_BUF_HOST) return 0;
    o->device = static_cast<uint8_t *>(g_staging.base) + off;
    off += (o->bytes + 255) / 256 * 256;
    if (copy_in && cudaMemcpy(o->device, o->host, o->bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ELAUNCH;
    }
    return 0;
  };
  for (auto *o : inputs)
    if (int rc = place(o, true)) return rc;
  for (auto *o : outputs)
    if (int rc = place(o, false)) return rc;
  return 0;
}

int stage_out(std::vector<Operand *> outputs) {
  for (auto *o : outputs) {
    if (!o || !o->present || o->buf.kind != HTPG_BUF_HOST) continue;
    if (cudaMemcpy(o->host, o->device, o->bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ELAUNCH;
    }
  }
  return 0;
}

// Prepared weight for a {fd, offset} weight operand.  Host-memory blobs are
// copied to the device once per (fd, offset, generation).
// qtype (opcodes 2-4): the ggml type of a super-block stream (int8 unused).
int exec_weights(const Operand &o, bool int8, int k, int n, htpg_weights **out, int qtype = 0) {
  const WeightKey key(o.fd, o.offset, o.buf.generation, qtype ? 100 + qtype : int8 ? 0 : 1, k, n);
  {
    std::lock_guard<std::recursive_mutex> lk(g_reg_mu);
    auto it = g_exec_weights.find(key);
    if (it != g_exec_weights.end()) {
      *out = it->second;
      return 0;
    }
  }
  const void *src = o.host;
  void *tmp = nullptr;
  if (o.buf.kind == HTPG_BUF_HOST) {
    if (cudaMalloc(&tmp, o.bytes) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ENOMEM;
    }
    if (cudaMemcpy(tmp, o.host, o.bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaGetLastError();
      cudaFree(tmp);
      return HTPG_ELAUNCH;
    }
    src = tmp;
  }
  htpg_weights *w = nullptr;
  const int rc = qtype ? htpg_qk0_weights_create(src, k, n, qtype, nullptr, &w)
                 : int8 ? htpg_w8a8_weights_create(src, k, n, 0, 0, nullptr, &w)
                        : htpg_f16_weights_create(static_cast<const uint16_t *>(src), k, n, 0, 0, nullptr, &w);
  if (tmp) cudaFree(tmp);
  if (rc) return rc;
  std::lock_guard<std::recursive_mutex> lk(g_reg_mu);
  g_exec_weights[key] = w;
  *out = w;
  return 0;
}

uint64_t fnv1a(const void *data, size_t size) {
  const uint8_t *p = static_cast<const uint8_t *>(data);
  uint64_t h = 14695981039346656037ull;
  if (!p) return 0;
  for (size_t i = 0; i < size; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

// FNV-1a of an operand as the device sees it (host copy for device buffers).
uint64_t operand_hash(const void *device, size_t bytes) {
  std::vector<uint8_t> tmp(bytes);
  if (cudaMemcpy(tmp.data(), device, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return fnv1a(tmp.data(), bytes);
}

bool checked_mul(size_t a, size_t b, size_t *r) {
  if (a != 0 && b > SIZE_MAX / a) return false;
  *r = a * b;
  return true;
}

typedef std::chrono::steady_clock Clock;
int32_t elapsed_us(Clock::time_point t0) {
  return static_cast<int32_t>(std::chrono::duration_cast<std::chrono::microseconds>(Clock::now() - t0).count());
}

int sync_status(int rc) {
  if (rc) return rc;
  return htpg_check_device(nullptr, nullptr);
}

// Host-memory activation and output: rows go through in chunks on three
// streams (copy in, GEMM, copy out, ordered per chunk by events) so that the
// copies of different chunks overlap each other and the GEMMs; PCIe carries
// both directions at once.  Returns the first error.
struct ChunkStreams {
  bool ready = false;
  cudaStream_t in = nullptr, cmp = nullptr, out = nullptr;
  std::vector<cudaEvent_t> ev;  // 2 per chunk
};
ChunkStreams g_chunk;

int w8a8_chunked(htpg_weights *w, Operand &out, Operand &act, Operand &bias, int m, int k, int n, int channels,
                 int mode) {
  if (!g_chunk.ready) {
    if (cudaStreamCreateWithFlags(&g_chunk.in, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&g_chunk.cmp, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&g_chunk.out, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ELAUNCH;
    }
    g_chunk.ready = true;
  }
  const int chunks_target = 12;
  int rows = (m + chunks_target - 1) / chunks_target;
  rows = (rows + 127) / 128 * 128;
  const int chunks = (m + rows - 1) / rows;
  while (static_cast<int>(g_chunk.ev.size()) < 2 * chunks) {
    cudaEvent_t e;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ELAUNCH;
    }
    g_chunk.ev.push_back(e);
  }
  const uint8_t *xh = static_cast<const uint8_t *>(act.host);
  uint8_t *xd = static_cast<uint8_t *>(act.device);
  uint8_t *oh = static_cast<uint8_t *>(out.host);
  uint8_t *od = static_cast<uint8_t *>(out.device);
  int rc = 0;
  for (int c = 0; c < chunks && !rc; ++c) {
    const int r0 = c * rows, nr = std::min(rows, m - r0);
    const size_t xoff = static_cast<size_t>(r0) * k * 4, xbytes = static_cast<size_t>(nr) * k * 4;
    const size_t ooff = static_cast<size_t>(r0) * n * 4, obytes = static_cast<size_t>(nr) * n * 4;
    cudaEvent_t e_in = g_chunk.ev[2 * c], e_cmp = g_chunk.ev[2 * c + 1];
    if (cudaMemcpyAsync(xd + xoff, xh + xoff, xbytes, cudaMemcpyHostToDevice, g_chunk.in) != cudaSuccess ||
        cudaEventRecord(e_in, g_chunk.in) != cudaSuccess || cudaStreamWaitEvent(g_chunk.cmp, e_in, 0) != cudaSuccess) {
      cudaGetLastError();
      rc = HTPG_ELAUNCH;
      break;
    }
    rc = htpg_w8a8_run(w, reinterpret_cast<float *>(od + ooff), n, reinterpret_cast<const float *>(xd + xoff),
                       bias.present ? static_cast<const float *>(bias.device) : nullptr, nr, channels, mode,
                       g_chunk.cmp);
    if (rc) break;
    if (cudaEventRecord(e_cmp, g_chunk.cmp) != cudaSuccess || cudaStreamWaitEvent(g_chunk.out, e_cmp, 0) != cudaSuccess ||
        cudaMemcpyAsync(oh + ooff, od + ooff, obytes, cudaMemcpyDeviceToHost, g_chunk.out) != cudaSuccess) {
      cudaGetLastError();
      rc = HTPG_ELAUNCH;
    }
  }
  const cudaError_t e1 = cudaStreamSynchronize(g_chunk.in), e2 = cudaStreamSynchronize(g_chunk.cmp),
                    e3 = cudaStreamSynchronize(g_chunk.out);
  if (!rc && (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess)) {
    cudaGetLastError();
    rc = HTPG_ELAUNCH;
  }
  return rc ? rc : htpg_check_device(nullptr, nullptr);
}

// ---- opcode 15: native W8A8 linear (op_executor.cc:314-353) -----------------
int exec_w8a8(uint8_t *payload, size_t payload_size) {
  const bool profiled = payload_size == sizeof(NativeW8A8ProfileParams);
  const bool cpu = payload_size == sizeof(NativeW8A8CpuParams);
  const bool epi = payload_size == sizeof(NativeW8A8EpilogueParams);
  if (payload_size != sizeof(NativeW8A8Params) && !profiled && !cpu && !epi) return -1;
  NativeW8A8Params *p = reinterpret_cast<NativeW8A8Params *>(payload);
  const int m = p->m, k = p->k, n = p->n;
  if (m < 1 || m > HTPG_W8A8_MAX_M || k < 32 || k > HTPG_W8A8_MAX_K || k % 32 || n < 64 ||
      n > HTPG_W8A8_MAX_N || n % 64)
    return -1;
  int mode = 0, channels = n;
  RpcmemBufAddr bias_addr = {-1, 0};
  if (epi) {
    const NativeW8A8EpilogueParams *e = reinterpret_cast<NativeW8A8EpilogueParams *>(payload);
    mode = e->mode;
    channels = e->channels;
    bias_addr = e->bias;
    if (mode < 0 || mode > 3 || channels < 1 || channels > n || (mode != 3 && channels != n)) return -1;
  }
  const size_t constants_size = 128u + static_cast<size_t>(k) * n + static_cast<size_t>(n) * 8 +
                                static_cast<size_t>(k) * 4;
  const size_t out_cols = mode == 3 ? static_cast<size_t>(channels) : static_cast<size_t>(n);
  Operand out, act, cst, ctl, bias;
  const int r0 = resolve(out, p->output.fd, p->output.offset, static_cast<size_t>(m) * out_cols * 4);
  const int r1 = resolve(act, p->activation.fd, p->activation.offset, static_cast<size_t>(m) * k * 4);
  const int r2 = resolve(cst, p->constants.fd, p->constants.offset, constants_size);
  if (r0 || r1 || r2) return -2;
  if (cpu) {
    const NativeW8A8CpuParams *c = reinterpret_cast<NativeW8A8CpuParams *>(payload);
    if (resolve(ctl, c->control.fd, c->control.offset, sizeof(W8A8CpuControl))) return -2;
  }
  if (epi && bias_addr.fd >= 0 &&
      resolve(bias, bias_addr.fd, bias_addr.offset, static_cast<size_t>(channels) * 4))
    return -2;
  // header check on the caller-visible bytes (op_executor.cc:331-335)
  W8A8Header h;
  if (cst.buf.kind == HTPG_BUF_HOST) {
    std::memcpy(&h, cst.host, sizeof(h));
  } else if (cudaMemcpy(&h, cst.host, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return HTPG_ELAUNCH;
  }
  const size_t kn = static_cast<size_t>(k) * n;
  if (h.magic != W8A8_HEADER_MAGIC || h.version != 1 || h.k != static_cast<uint32_t>(k) ||
      h.n != static_cast<uint32_t>(n) || h.weight_offset != 128 || h.scale_offset != 128u + kn ||
      h.sum_offset != h.scale_offset + 4u * n || h.inverse_offset != h.sum_offset + 4u * n ||
      h.bytes != constants_size)
    return -3;
  NativeW8A8Profile prof;
  std::memset(&prof, 0, sizeof(prof));
  if (profiled) {
    std::memcpy(&prof, payload + sizeof(NativeW8A8Params), sizeof(prof));
    if (prof.mode != 1 && prof.mode != 2 && prof.mode != 3) return -1;
  }
  if (cpu) {
    // CPU-epilogue form (linear_w8a8.c:512-526): raw byte planes into the
    // output tensor, row scales and the batch descriptor into the control block
    if (m > 4096) return -10;
    htpg_weights *w = nullptr;
    int rc = exec_weights(cst, true, k, n, &w);
    if (rc) return rc;
    if ((rc = stage_in({&act}, {&out}))) return rc;
    W8A8CpuControl *control = static_cast<W8A8CpuControl *>(ctl.host);
    std::vector<uint8_t> ctl_copy;
    if (ctl.buf.kind == HTPG_BUF_DEVICE) {  // the control block lives in HBM: work on a host copy
      ctl_copy.resize(sizeof(W8A8CpuControl));
      if (cudaMemcpy(ctl_copy.data(), ctl.device, ctl_copy.size(), cudaMemcpyDeviceToHost) != cudaSuccess) {
        cudaGetLastError();
        return HTPG_ELAUNCH;
      }
      control = reinterpret_cast<W8A8CpuControl *>(ctl_copy.data());
    }
    const auto t0 = Clock::now();
    rc = htpg_w8a8_run_planes(w, static_cast<float *>(out.device), static_cast<const float *>(act.device), m,
                              control, nullptr);
    p->elapsed_us = elapsed_us(t0);
    if (rc) return rc;
    if ((rc = stage_out({&out}))) return rc;
    if (!ctl_copy.empty() &&
        cudaMemcpy(ctl.device, ctl_copy.data(), ctl_copy.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ELAUNCH;
    }
    return 0;
  }
  htpg_weights *w = nullptr;
  const auto t_setup = Clock::now();
  int rc = exec_weights(cst, true, k, n, &w);
  if (rc) return rc;
  const double setup_ms = std::chrono::duration<double, std::milli>(Clock::now() - t_setup).count();
  if (!profiled && mode != 3 && m >= 1024 && act.buf.kind == HTPG_BUF_HOST && out.buf.kind == HTPG_BUF_HOST) {
    // the activation gets a device region here and is copied chunk by chunk
    if ((rc = stage_in({&bias}, {&act, &out}))) return rc;
    const auto t0 = Clock::now();
    rc = w8a8_chunked(w, out, act, bias, m, k, n, channels, mode);
    p->elapsed_us = elapsed_us(t0);
    return rc;
  }
  if ((rc = stage_in({&act, &bias}, {&out}))) return rc;
  const auto t0 = Clock::now();
  if (profiled) htpg_set_profiling(1);
  rc = htpg_w8a8_run(w, static_cast<float *>(out.device), 0, static_cast<const float *>(act.device),
                     bias.present ? static_cast<const float *>(bias.device) : nullptr, m, channels, mode,
                     nullptr);
  rc = sync_status(rc);
  if (profiled) htpg_set_profiling(0);
  p->elapsed_us = elapsed_us(t0);
  if (profiled) {
    // the trailer is written back like the reference's (op_executor.cc:344-346)
    htpg_w8a8_profile_fill(m, k, n, setup_ms, &prof);
    std::memcpy(payload + sizeof(NativeW8A8Params), &prof, sizeof(prof));
  }
  if (rc) return rc;
  return stage_out({&out});
}

// ---- opcode 16: packed FP16 GEMM + epilogue (op_executor.cc:446-471) ----------
int exec_f16_epilogue(uint8_t *payload, size_t payload_size) {
  if (payload_size != sizeof(F16EpilogueParams)) return -1;
  F16EpilogueParams *p = reinterpret_cast<F16EpilogueParams *>(payload);
  if (p->m <= 0 || p->k <= 0 || p->n <= 0 || p->k % 32 || p->n % 32 || p->channels <= 0 ||
      p->channels > p->n || p->mode < 0 || p->mode > 3 || (p->mode != 3 && p->channels != p->n))
    return -1;
  size_t out_size, act_size, w_size;
  if (!checked_mul(static_cast<size_t>(p->m), static_cast<size_t>(p->channels) * 4, &out_size) ||
      !checked_mul(static_cast<size_t>(p->m), static_cast<size_t>(p->k) * 4, &act_size) ||
      !checked_mul(static_cast<size_t>(p->k), static_cast<size_t>(p->n) * 2, &w_size))
    return -1;
  Operand out, act, wt, bias;
  if (resolve(out, p->output.fd, p->output.offset, out_size) ||
      resolve(act, p->activation.fd, p->activation.offset, act_size) ||
      resolve(wt, p->weight.fd, p->weight.offset, w_size))
    return -1;
  if (p->bias.fd >= 0 && resolve(bias, p->bias.fd, p->bias.offset, static_cast<size_t>(p->channels) * 4))
    return -1;
  htpg_weights *w = nullptr;
  int rc = exec_weights(wt, false, p->k, p->n, &w);
  if (rc) return rc;
  if ((rc = stage_in({&act, &bias}, {&out}))) return rc;
  const auto t0 = Clock::now();
  rc = htpg_f16_run(w, static_cast<float *>(out.device), 0, static_cast<const float *>(act.device),
                    bias.present ? static_cast<const float *>(bias.device) : nullptr, p->m, p->channels,
                    p->mode, nullptr);
  rc = sync_status(rc);
  p->elapsed_us = elapsed_us(t0);
  if (rc) return rc;
  return stage_out({&out});
}

// ---- opcode 17: packed-FP16 NCHW convolution (op_executor.cc:405-425) ----------
int exec_conv(uint8_t *payload, size_t payload_size) {
  if (payload_size != sizeof(NativeConvParams)) return -1;
  NativeConvParams *p = reinterpret_cast<NativeConvParams *>(payload);
  if (p->iw <= 0 || p->ih <= 0 || p->ic <= 0 || p->oc <= 0 || p->batch <= 0 || p->ow <= 0 || p->oh <= 0 ||
      p->kw <= 0 || p->kh <= 0 || p->sx <= 0 || p->sy <= 0 || p->dx <= 0 || p->dy <= 0 || p->kp % 32 ||
      p->np % 32 || p->np < p->oc || p->kp < static_cast<int64_t>(p->kw) * p->kh * p->ic ||
      (p->upscale != 1 && p->upscale != 2) ||
      p->ow != (p->upscale * p->iw + 2 * p->px - p->dx * (p->kw - 1) - 1) / p->sx + 1 ||
      p->oh != (p->upscale * p->ih + 2 * p->py - p->dy * (p->kh - 1) - 1) / p->sy + 1)
    return -1;
  const size_t in_size = static_cast<size_t>(p->iw) * p->ih * p->ic * p->batch * 4;
  const size_t out_size = static_cast<size_t>(p->ow) * p->oh * p->oc * p->batch * 4;
  const size_t w_size = static_cast<size_t>(p->kp) * p->np * 2;
  if (in_size > INT32_MAX || out_size > INT32_MAX || w_size > INT32_MAX) return -1;
  Operand out, act, wt, bias;
  if (resolve(out, p->output.fd, p->output.offset, out_size) ||
      resolve(act, p->activation.fd, p->activation.offset, in_size) ||
      resolve(wt, p->weight.fd, p->weight.offset, w_size))
    return -1;
  if (p->bias.fd >= 0 && resolve(bias, p->bias.fd, p->bias.offset, static_cast<size_t>(p->oc) * 4)) return -1;
  const auto t0 = Clock::now();
  htpg_weights *w = nullptr;
  int rc = exec_weights(wt, false, p->kp, p->np, &w);
  if (rc) return rc;
  const int32_t weight_us = elapsed_us(t0);
  if ((rc = stage_in({&act, &bias}, {&out}))) return rc;
  rc = htpg_conv2d_run(w, static_cast<float *>(out.device), static_cast<const float *>(act.device),
                       bias.present ? static_cast<const float *>(bias.device) : nullptr, p, nullptr);
  rc = sync_status(rc);
  p->elapsed_us = elapsed_us(t0);
  // im2col and GEMM run back to back on the device; the epilogue is fused
  p->weight_us = weight_us;
  p->gather_us = 0;
  p->hmx_us = p->elapsed_us - weight_us;
  p->store_us = 0;
  if (rc) return rc;
  return stage_out({&out});
}

// ---- opcode 19: FP32 model auxiliaries (op_executor.cc:371-401) -------------
int exec_aux(uint8_t *payload, size_t payload_size) {
  if (payload_size != sizeof(NativeAuxParams)) return -1;
  NativeAuxParams *p = reinterpret_cast<NativeAuxParams *>(payload);
  if (htpg_model_aux_check(p, p->weight.fd >= 0, p->bias.fd >= 0) != HTPG_OK) return -1;
  const int n = p->mode == 2 ? p->channels : p->mode == 9 ? p->other_count : p->mode == 10 ? p->count : p->width;
  size_t input_bytes = static_cast<size_t>(p->count) * 4;
  if (p->mode == 12 || p->mode == 13)
    input_bytes = (static_cast<size_t>(p->spatial) * p->batch - 1) * p->channels * 4 + static_cast<size_t>(2) * p->width * 4;
  Operand out, in, w, b;
  if (resolve(out, p->output.fd, p->output.offset, static_cast<size_t>(p->count) * 4) ||
      resolve(in, p->input.fd, p->input.offset, input_bytes))
    return -1;
  if (p->weight.fd >= 0 && resolve(w, p->weight.fd, p->weight.offset, static_cast<size_t>(p->other_count) * 4))
    return -1;
  if (p->bias.fd >= 0 && resolve(b, p->bias.fd, p->bias.offset, static_cast<size_t>(n) * 4)) return -1;
  int rc = stage_in({&in, &w, &b}, {&out});
  if (rc) return rc;
  const auto t0 = Clock::now();
  rc = htpg_model_aux(static_cast<float *>(out.device), static_cast<const float *>(in.device),
                      w.present ? static_cast<const float *>(w.device) : nullptr,
                      b.present ? static_cast<const float *>(b.device) : nullptr, p, nullptr);
  rc = sync_status(rc);
  p->elapsed_us = elapsed_us(t0);
  if (rc) return rc;
  return stage_out({&out});
}

// ---- opcode 1: packed FP16 GEMM, no epilogue (op_executor.cc:473-540) ----------
bool op_trace_enabled() { return std::getenv("HTPG_OP_TRACE") != nullptr; }

int exec_w16a32(uint8_t *payload, size_t payload_size) {
  if (payload_size < sizeof(MatMulParams)) return -1;
  MatMulParams *p = reinterpret_cast<MatMulParams *>(payload);
  const int m = p->m, k = p->k, n = p->n;
  if (m <= 0 || k <= 0 || n <= 0) return -10;
  Operand out, act, wt;
  if (resolve(out, p->output.fd, p->output.offset, static_cast<size_t>(m) * n * 4) ||
      resolve(act, p->activation.fd, p->activation.offset, static_cast<size_t>(m) * k * 4) ||
      resolve(wt, p->weight.fd, p->weight.offset, static_cast<size_t>(k) * n * 2))
    return -2;
  if ((reinterpret_cast<uintptr_t>(out.host) | reinterpret_cast<uintptr_t>(act.host) |
       reinterpret_cast<uintptr_t>(wt.host)) & 127u)
    return -3;
  if (k % 32 || n % 32) return -11;
  htpg_weights *w = nullptr;
  int rc = exec_weights(wt, false, k, n, &w);
  if (rc) return rc;
  if ((rc = stage_in({&act}, {&out}))) return rc;
  const bool trace = op_trace_enabled();
  if (trace) {
    p->debug_vtcm_base = 0;
    p->debug_vtcm_size = 0;
    p->debug_vtcm_ctx = 0;
    p->debug_hmx_ctx = 0;
    p->debug_worker_pool = 0;
    p->debug_hmx_lock_result = 0;
    p->debug_dsp_activation_hash = operand_hash(act.device, act.bytes);
  }
  const auto t0 = Clock::now();
  rc = htpg_f16_run(w, static_cast<float *>(out.device), 0, static_cast<const float *>(act.device), nullptr,
                    m, n, 0, nullptr);
  rc = sync_status(rc);
  if (payload_size >= sizeof(MatMulProfileParams))
    reinterpret_cast<MatMulProfileParams *>(payload)->elapsed_us = elapsed_us(t0);
  if (rc) return rc;
  rc = stage_out({&out});
  if (trace) {
    p->debug_dsp_output_hash = operand_hash(out.device, out.bytes);
    p->debug_dsp_output_hash_after_invalidate =
        out.buf.kind == HTPG_BUF_HOST ? fnv1a(out.host, out.bytes) : p->debug_dsp_output_hash;
  }
  return rc;
}

// ---- opcodes 2-4: ggml-block weight GEMMs (op_executor.cc:771-808) ----------
// MatMulParams payload (at least 92 bytes; 96 with elapsed_us); the weight
// operand is k*n/256 super-blocks of the opcode's type, prepared once per
// {fd, offset, generation} like the other weights.  Kernel-level checks
// (mat_mul.c:1604-1613) answer -1.
int exec_qk0(int op, uint8_t *payload, size_t payload_size) {
  if (payload_size < sizeof(MatMulParams)) return -1;
  const int qt = op == HTP_OPS_MAT_MUL_PERMUTED_W4D16A32   ? HTPG_GGML_Q4_0
                 : op == HTP_OPS_MAT_MUL_PERMUTED_W8D16A32 ? HTPG_GGML_Q8_0
                                                           : HTPG_GGML_IQ4_NL;
  MatMulParams *p = reinterpret_cast<MatMulParams *>(payload);
  const int m = p->m, k = p->k, n = p->n;
  if (m <= 0 || k <= 0 || n <= 0) return -1;
  const size_t wbytes = static_cast<size_t>(k) * static_cast<size_t>(n) / 256u *
                        (qt == HTPG_GGML_Q8_0 ? 272u : 144u);
  Operand out, act, wt;
  if (resolve(out, p->output.fd, p->output.offset, static_cast<size_t>(m) * n * 4) ||
      resolve(act, p->activation.fd, p->activation.offset, static_cast<size_t>(m) * k * 4) ||
      resolve(wt, p->weight.fd, p->weight.offset, wbytes))
    return -2;
  if (k % 32 || n % 32) return -1;
  if ((reinterpret_cast<uintptr_t>(out.host) | reinterpret_cast<uintptr_t>(act.host) |
       reinterpret_cast<uintptr_t>(wt.host)) & 127u)
    return -1;
  htpg_weights *w = nullptr;
  int rc = exec_weights(wt, false, k, n, &w, qt);  // stage records, made once per {fd, offset, generation}
  if (rc) return rc;
  if ((rc = stage_in({&act}, {&out}))) return rc;
  const auto t0 = Clock::now();
  rc = htpg_qk0_run(w, static_cast<float *>(out.device), static_cast<const float *>(act.device), m, nullptr);
  rc = sync_status(rc);
  if (payload_size >= sizeof(MatMulProfileParams))
    reinterpret_cast<MatMulProfileParams *>(payload)->elapsed_us = elapsed_us(t0);
  if (rc) return rc;
  return stage_out({&out});
}

}  // namespace

extern "C" int execute_op_simple(struct OpComputeRequest *req, size_t req_size) {
  if (!req || req_size < sizeof(OpComputeRequest)) return -1;
  const size_t payload_size = req_size - sizeof(OpComputeRequest);
  std::lock_guard<std::mutex> lk(g_exec_mu);
  switch (req->op) {
    case HTP_OPS_MAT_MUL_NATIVE_W8A8: return exec_w8a8(req->payload, payload_size);
    case HTP_OPS_MAT_MUL_F16_EPILOGUE: return exec_f16_epilogue(req->payload, payload_size);
    case HTP_OPS_MAT_MUL_PERMUTED_W16A32: return exec_w16a32(req->payload, payload_size);
    case HTP_OPS_CONV2D_NCHW_F16: return exec_conv(req->payload, payload_size);
    case HTP_OPS_MODEL_AUX_F32: return exec_aux(req->payload, payload_size);
    case HTP_OPS_MAT_MUL_PERMUTED_W4D16A32:
    case HTP_OPS_MAT_MUL_PERMUTED_W8D16A32:
    case HTP_OPS_MAT_MUL_PERMUTED_W4D16A32_IQ4_NL: return exec_qk0(req->op, req->payload, payload_size);
    default:
      // Registered opcodes outside this library's path are refused so the
      // caller keeps them on its own backend; unknown opcodes are ignored with
      // state 0, as the reference dispatcher does (op_executor.cc:1104-1106).
      return req->op < HTP_OPS_COUNT ? AEE_EUNSUPPORTED : 0;
  }
}

// ================================================================ backends
namespace {

struct Backend;

struct Channel {
  uint8_t *msg = nullptr;
  int fd = -1;
  size_t max_msg_size = 0;
  uint64_t token = 0;
  std::atomic<bool> stop{false};
  std::thread thread;
};

struct Backend {
  bool opened = false;
  bool initialized = false;
  bool mapping_only = false;
  int device = 0;
  uint32_t fraction_num = 1, fraction_den = 1;
  Channel chan;
};

std::mutex g_be_mu;
std::mutex g_live_mu;
std::set<Backend *> g_live;  // handles returned by htp_ops_open and not yet closed

// Resolve a handle; stale or foreign handles give nullptr instead of a
// dangling object.
Backend *backend_of(remote_handle64 h) {
  Backend *b = reinterpret_cast<Backend *>(static_cast<uintptr_t>(h));
  std::lock_guard<std::mutex> lk(g_live_mu);
  return (b && g_live.count(b) && b->opened) ? b : nullptr;
}

// The 8 state bytes sit at offset 0 of the channel buffer (8-byte aligned).
inline uint64_t *state_word(uint8_t *msg) { return reinterpret_cast<uint64_t *>(msg); }
inline uint64_t load_acquire(uint64_t *p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void store_release(uint64_t *p, uint64_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }

// RPCMEM map request: "gets" must name registered buffers; "puts" drop what
// this library derived from the buffer (cached weight repacks).  commu.c:187-246.
int handle_map_request(Channel &c, uint8_t *data, size_t size) {
  if (size < sizeof(RpcmemMapRequest)) return -1;
  const bool v2 = size >= sizeof(RpcmemMapRequestV2) &&
                  reinterpret_cast<RpcmemMapRequestV2 *>(data)->magic == RPCMEM_MAP_REQUEST_SESSION_MAGIC &&
                  reinterpret_cast<RpcmemMapRequestV2 *>(data)->version == RPCMEM_MAP_REQUEST_VERSION_SESSION;
  if (v2) {
    RpcmemMapRequestV2 *r = reinterpret_cast<RpcmemMapRequestV2 *>(data);
    const size_t avail = (size - sizeof(*r)) / sizeof(RpcmemMapEntryV2);
    if (r->header_size < sizeof(*r) || r->n_puts < 0 || r->n_gets < 0 || r->session_token != c.token)
      return -1;
    if (static_cast<size_t>(r->n_puts) + static_cast<size_t>(r->n_gets) > avail) return -1;
    for (int j = 0; j < r->n_puts; ++j)
      if (htpg_buffer_touch(r->entries[j].fd) != HTPG_OK) return -1;
    for (int j = 0; j < r->n_gets; ++j) {
      const RpcmemMapEntryV2 &e = r->entries[r->n_puts + j];
      if (!htpg_buffer_resolve(e.fd, static_cast<int64_t>(e.offset), e.size, nullptr)) return -1;
    }
    return 0;
  }
  RpcmemMapRequest *r = reinterpret_cast<RpcmemMapRequest *>(data);
  const size_t avail = (size - sizeof(*r)) / sizeof(int32_t);
  if (r->n_puts < 0 || r->n_gets < 0 || static_cast<size_t>(r->n_puts) > avail ||
      static_cast<size_t>(r->n_gets) > avail - static_cast<size_t>(r->n_puts))
    return -1;
  for (int j = 0; j < r->n_puts; ++j) htpg_buffer_touch(r->fds[j]);
  return 0;
}

void receiver_loop(Backend *b) {
  Channel &c = b->chan;
  cudaSetDevice(b->device);
  MessageHeader *hdr = reinterpret_cast<MessageHeader *>(c.msg);
  unsigned idle = 0;
  while (!c.stop.load(std::memory_order_relaxed)) {
    const uint64_t d = load_acquire(state_word(c.msg));
    const uint8_t v0 = d & 0xff, v1 = (d >> 8) & 0xff;
    if (v0 == 0 || v1 != 0) {
      // spin briefly for latency, then back off like the reference's 1 us sleep
      if (++idle < 2048)
        std::this_thread::yield();
      else
        std::this_thread::sleep_for(std::chrono::microseconds(1));
      continue;
    }
    idle = 0;
    size_t total = 0;
    if (message_header_validate_layout(hdr, c.max_msg_size, &total)) {
      for (int i = 0; i < hdr->n_reqs; ++i) {
        const size_t wire = static_cast<size_t>(hdr->req_offsets[i + 1]) - static_cast<size_t>(hdr->req_offsets[i]);
        const size_t data_size = wire - sizeof(RequestHeader);
        RequestHeader *rq = message_header_get_request_ptr(hdr, i);
        switch (rq->type) {
          case REQUEST_TYPE_OP_COMPUTE:
            rq->state = b->mapping_only || !b->initialized
                            ? AEE_EBADSTATE
                            : execute_op_simple(reinterpret_cast<OpComputeRequest *>(rq->data), data_size);
            break;
          case REQUEST_TYPE_RPCMEM_MAP:
            rq->state = handle_map_request(c, rq->data, data_size);
            break;
          default:
            break;
        }
      }
    } else if (std::getenv("HTPG_LOG")) {
      std::fprintf(stderr, "htpg: invalid message layout n_reqs=%d capacity=%zu\n", hdr->n_reqs,
                   c.max_msg_size);
    }
    store_release(state_word(c.msg), static_cast<uint64_t>(v0) | (1ull << 8));
  }
}

AEEResult require_initialized(Backend *b) {
  if (!b || !b->initialized) return AEE_EBADSTATE;
  return AEE_SUCCESS;
}

AEEResult create_channel_internal(Backend *b, int32_t fd, uint32_t size, uint64_t token) {
  if (AEEResult r = require_initialized(b)) return r;
  if (b->chan.msg) return AEE_EALREADY;
  int kind = -1;
  void *p = htpg_buffer_resolve(fd, 0, size, &kind);
  if (!p || kind != HTPG_BUF_HOST || size < sizeof(MessageHeader) + sizeof(int32_t)) return -1;
  std::memset(p, 0, size);
  b->chan.msg = static_cast<uint8_t *>(p);
  b->chan.fd = fd;
  b->chan.max_msg_size = size;
  b->chan.token = token;
  b->chan.stop = false;
  b->chan.thread = std::thread(receiver_loop, b);
  return AEE_SUCCESS;
}

AEEResult destroy_channel_internal(Backend *b) {
  if (!b->chan.msg) return AEE_SUCCESS;
  b->chan.stop = true;
  if (b->chan.thread.joinable()) b->chan.thread.join();
  b->chan.msg = nullptr;
  b->chan.fd = -1;
  b->chan.max_msg_size = 0;
  b->chan.token = 0;
  return AEE_SUCCESS;
}

}  // namespace

extern "C" AEEResult htp_ops_open(const char *uri, remote_handle64 *handle) {
  (void)uri;
  if (!handle) return AEE_EBADPARM;
  Backend *b = new Backend;
  b->opened = true;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    dev = 0;
  }
  b->device = dev;
  {
    std::lock_guard<std::mutex> lk(g_live_mu);
    g_live.insert(b);
  }
  *handle = static_cast<remote_handle64>(reinterpret_cast<uintptr_t>(b));
  return AEE_SUCCESS;
}

extern "C" AEEResult htp_ops_close(remote_handle64 handle) {
  Backend *b = backend_of(handle);
  if (!b) return AEE_EBADSTATE;
  destroy_channel_internal(b);
  {
    std::lock_guard<std::mutex> lk(g_live_mu);
    g_live.erase(b);
  }
  b->opened = false;
  b->initialized = false;
  delete b;
  return AEE_SUCCESS;
}

extern "C" AEEResult htp_ops_init_backend(remote_handle64 handle) {
  Backend *b = backend_of(handle);
  if (!b) return AEE_EBADSTATE;
  if (b->initialized && !b->mapping_only) return AEE_SUCCESS;
  const int rc = htpg_init(b->device);
  if (rc == HTPG_ENOMEM) return AEE_ENOMEMORY;
  if (rc != HTPG_OK) return AEE_EFAILED;
  b->initialized = true;
  b->mapping_only = false;
  return AEE_SUCCESS;
}

extern "C" AEEResult htp_ops_init_backend_fraction(remote_handle64 handle, uint32_t numerator,
                                                   uint32_t denominator) {
  Backend *b = backend_of(handle);
  if (!b) return AEE_EBADSTATE;
  if (b->initialized) return AEE_SUCCESS;
  if (numerator == 0 || denominator == 0 || numerator > denominator) return AEE_EBADPARM;
  // VTCM shares have no device counterpart; the fraction is recorded only
  b->fraction_num = numerator;
  b->fraction_den = denominator;
  return htp_ops_init_backend(handle);
}

extern "C" AEEResult htp_ops_init_mapping_backend(remote_handle64 handle) {
  Backend *b = backend_of(handle);
  if (!b) return AEE_EBADSTATE;
  if (b->initialized) return AEE_SUCCESS;
  b->initialized = true;
  b->mapping_only = true;
  return AEE_SUCCESS;
}

extern "C" AEEResult htp_ops_release_backend(remote_handle64 handle) {
  Backend *b = backend_of(handle);
  if (!b) return AEE_EBADSTATE;
  b->initialized = false;
  b->mapping_only = true;
  return AEE_SUCCESS;
}

extern "C" AEEResult htp_ops_create_channel(remote_handle64 handle, int32_t fd, uint32_t size) {
  std::lock_guard<std::mutex> lk(g_be_mu);
  return create_channel_internal(backend_of(handle), fd, size, 0);
}

extern "C" AEEResult htp_ops_create_channel_with_token(remote_handle64 handle, uint64_t token, int32_t fd,
                                                       uint32_t size) {
  std::lock_guard<std::mutex> lk(g_be_mu);
  return create_channel_internal(backend_of(handle), fd, size, token);
}

extern "C" AEEResult htp_ops_destroy_channel(remote_handle64 handle) {
  std::lock_guard<std::mutex> lk(g_be_mu);
  Backend *b = backend_of(handle);
  if (!b) return AEE_EBADSTATE;
  return destroy_channel_internal(b);
}

extern "C" AEEResult htp_ops_rms_norm_f32(remote_handle64 handle, int32_t, int32_t, int32_t, int32_t,
                                          int32_t, int32_t) {
  if (AEEResult r = require_initialized(backend_of(handle))) return r;
  return AEE_EUNSUPPORTED;
}

namespace {

AEEResult direct_w16a32(remote_handle64 handle, int32_t ofd, int32_t ooff, int32_t afd, int32_t aoff,
                        int32_t wfd, int32_t woff, int32_t m, int32_t k, int32_t n, uint64_t *ahash,
                        uint64_t *ohash, uint64_t *ohash2) {
  Backend *b = backend_of(handle);
  if (AEEResult r = require_initialized(b)) return r;
  if (ahash) *ahash = 0;
  if (ohash) *ohash = 0;
  if (ohash2) *ohash2 = 0;
  if (m <= 0 || k <= 0 || n <= 0) return -10;
  cudaSetDevice(b->device);
  std::lock_guard<std::mutex> lk(g_exec_mu);
  Operand out, act, wt;
  if (resolve(out, ofd, ooff, static_cast<size_t>(m) * n * 4) ||
      resolve(act, afd, aoff, static_cast<size_t>(m) * k * 4) ||
      resolve(wt, wfd, woff, static_cast<size_t>(k) * n * 2))
    return AEE_EBADPARM;
  if (k % 32 || n % 32) return -11;
  htpg_weights *w = nullptr;
  int rc = exec_weights(wt, false, k, n, &w);
  if (rc) return rc;
  if ((rc = stage_in({&act}, {&out}))) return rc;
  if (ahash) *ahash = operand_hash(act.device, act.bytes);
  rc = sync_status(htpg_f16_run(w, static_cast<float *>(out.device), 0,
                                static_cast<const float *>(act.device), nullptr, m, n, 0, nullptr));
  if (rc) return rc;
  if (ohash) *ohash = operand_hash(out.device, out.bytes);
  rc = stage_out({&out});
  if (ohash2) *ohash2 = out.buf.kind == HTPG_BUF_HOST ? fnv1a(out.host, out.bytes) : operand_hash(out.device, out.bytes);
  return rc;
}

}  // namespace

extern "C" AEEResult htp_ops_mat_mul_permuted_w16a32(remote_handle64 handle, int32_t output_fd,
                                                     int32_t output_offset, int32_t activation_fd,
                                                     int32_t activation_offset, int32_t weight_fd,
                                                     int32_t weight_offset, int32_t m, int32_t k,
                                                     int32_t n) {
  return direct_w16a32(handle, output_fd, output_offset, activation_fd, activation_offset, weight_fd,
                       weight_offset, m, k, n, nullptr, nullptr, nullptr);
}

extern "C" AEEResult htp_ops_mat_mul_permuted_w16a32_trace(remote_handle64 handle, int32_t output_fd,
                                                           int32_t output_offset, int32_t activation_fd,
                                                           int32_t activation_offset, int32_t weight_fd,
                                                           int32_t weight_offset, int32_t m, int32_t k,
                                                           int32_t n, uint64_t *activation_hash,
                                                           uint64_t *output_hash,
                                                           uint64_t *output_hash_after_remap) {
  return direct_w16a32(handle, output_fd, output_offset, activation_fd, activation_offset, weight_fd,
                       weight_offset, m, k, n, activation_hash, output_hash, output_hash_after_remap);
}

// Self-checks (reference: commu.c:813-827 runs on-device contract tests): the
// wire ABI sizes and one exact W8A8 product on the device.
extern "C" AEEResult htp_ops_test_ops(remote_handle64 handle, int32_t *userdma_scope) {
  Backend *b = backend_of(handle);
  if (AEEResult r = require_initialized(b)) return r;
  if (!userdma_scope) return AEE_EBADPARM;
  *userdma_scope = 0;
  if (sizeof(NativeW8A8Params) != 40 || sizeof(F16EpilogueParams) != 56 || sizeof(MatMulParams) != 92)
    return AEE_EFAILED;
  // 64 x 64 weight of +1 in column c's first c+1 inputs; x = one-hot rows
  const int m = 2, k = 64, n = 64;
  std::vector<int8_t> wnk(static_cast<size_t>(n) * k, 0);
  for (int c = 0; c < n; ++c)
    for (int r = 0; r <= c; ++r) wnk[static_cast<size_t>(c) * k + r] = 1;
  const size_t bytes = 128u + static_cast<size_t>(k) * n + 8u * n + 4u * k;
  std::vector<uint8_t> blob(bytes, 0);
  W8A8Header h;
  std::memset(&h, 0, sizeof(h));
  h.magic = W8A8_HEADER_MAGIC;
  h.version = 1;
  h.k = k;
  h.n = n;
  h.weight_offset = 128;
  h.scale_offset = 128 + k * n;
  h.sum_offset = h.scale_offset + 4 * n;
  h.inverse_offset = h.sum_offset + 4 * n;
  h.bytes = static_cast<uint32_t>(bytes);
  std::memcpy(blob.data(), &h, sizeof(h));
  for (int c = 0; c < n; ++c) {
    int32_t s = 0;
    for (int r = 0; r < k; ++r) {
      const size_t off = static_cast<size_t>(c / 64) * 64 * k + static_cast<size_t>(r / 32) * 2048 +
                         static_cast<size_t>((c % 64) / 32) * 1024 + static_cast<size_t>((r % 32) / 4) * 128 +
                         static_cast<size_t>(c % 32) * 4 + r % 4;
      blob[128 + off] = static_cast<uint8_t>(wnk[static_cast<size_t>(c) * k + r]);
      s += wnk[static_cast<size_t>(c) * k + r];
    }
    const float one = 1.0f;
    std::memcpy(blob.data() + h.scale_offset + 4 * c, &one, 4);
    std::memcpy(blob.data() + h.sum_offset + 4 * c, &s, 4);
  }
  for (int r = 0; r < k; ++r) {
    const float one = 1.0f;
    std::memcpy(blob.data() + h.inverse_offset + 4 * r, &one, 4);
  }
  std::vector<float> x(static_cast<size_t>(m) * k, 0.0f), out(static_cast<size_t>(m) * n, -1.0f);
  x[0] = 127.0f;       // row 0: input 0 -> code +127, scale 1
  x[k + 5] = -127.0f;  // row 1: input 5 -> code -127, scale 1
  void *dblob = nullptr, *dx = nullptr, *dout = nullptr;
  AEEResult result = AEE_EFAILED;
  cudaSetDevice(b->device);
  if (cudaMalloc(&dblob, bytes) == cudaSuccess && cudaMalloc(&dx, x.size() * 4) == cudaSuccess &&
      cudaMalloc(&dout, out.size() * 4) == cudaSuccess &&
      cudaMemcpy(dblob, blob.data(), bytes, cudaMemcpyHostToDevice) == cudaSuccess &&
      cudaMemcpy(dx, x.data(), x.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess) {
    const int rc = hmx_mat_mul_native_w8a8(static_cast<float *>(dout), static_cast<float *>(dx),
                                           static_cast<uint8_t *>(dblob), m, k, n);
    if (rc == 0 && cudaMemcpy(out.data(), dout, out.size() * 4, cudaMemcpyDeviceToHost) == cudaSuccess) {
      bool good = true;
      for (int c = 0; c < n; ++c) {
        good = good && out[c] == 127.0f;                          // every column uses input 0
        good = good && out[n + c] == (c >= 5 ? -127.0f : 0.0f);   // input 5 only in columns >= 5
      }
      result = good ? AEE_SUCCESS : AEE_EFAILED;
    }
  }
  cudaGetLastError();
  htpg_weight_cache_drop(dblob);
  cudaFree(dblob);
  cudaFree(dx);
  cudaFree(dout);
  return result;
}

// ================================================================ sessions
struct htp_ops_session {
  remote_handle64 handle = 0;
  uint32_t session_id = 0;
  uint32_t session_index = 0;
  uint32_t effective_domain_id = 0;
  int base_domain_id = 0;
  int reserved = 0;
  int backend_initialized = 0;
  int channel_initialized = 0;
};

namespace {

htp_ops_session *g_default_session = nullptr;
htp_ops_session *g_active_session = nullptr;
constexpr uint32_t kMaxReserved = 32;
int g_reserved_used[kMaxReserved] = {0};
uint32_t g_next_session_id = 1;

uint32_t alloc_reserved_index() {
  for (uint32_t i = 1; i < kMaxReserved; ++i)
    if (!g_reserved_used[i]) {
      g_reserved_used[i] = 1;
      return i;
    }
  return 0;
}

uint64_t session_token(const htp_ops_session *s) {
  if (!s || !s->reserved) return 0;
  return (static_cast<uint64_t>(s->session_index) << 32) | s->effective_domain_id;
}

}  // namespace

extern "C" int htp_ops_session_open(htp_ops_session **out, int base_domain, const char *name, int reserve_new) {
  if (!out) return -1;
  *out = nullptr;
  htp_ops_session *s = new htp_ops_session;
  s->base_domain_id = base_domain;
  s->effective_domain_id = static_cast<uint32_t>(base_domain);
  s->reserved = reserve_new != 0;
  s->session_id = g_next_session_id++;
  if (htp_ops_open(name, &s->handle) != AEE_SUCCESS) {
    delete s;
    return -1;
  }
  if (s->reserved) {
    s->session_index = alloc_reserved_index();
    if (s->session_index == 0) {
      htp_ops_close(s->handle);
      delete s;
      return -1;
    }
  }
  *out = s;
  return 0;
}

extern "C" htp_ops_session *htp_ops_default_session(void) { return g_default_session; }

extern "C" int htp_ops_session_init_backend(htp_ops_session *s) {
  if (!s || !s->handle) return -1;
  const char *multi = std::getenv("SD_HTP_MULTI_SESSION");
  const int err = (s->reserved && multi && multi[0] != '0') ? htp_ops_init_mapping_backend(s->handle)
                                                            : htp_ops_init_backend(s->handle);
  if (err == AEE_SUCCESS) s->backend_initialized = 1;
  return err;
}

extern "C" int htp_ops_session_acquire_backend(htp_ops_session *s) {
  if (!s || !s->handle) return -1;
  const int err = htp_ops_init_backend(s->handle);
  if (err == AEE_SUCCESS) s->backend_initialized = 1;
  return err;
}

extern "C" int htp_ops_session_release_backend(htp_ops_session *s) {
  if (!s || !s->handle) return -1;
  const int err = htp_ops_release_backend(s->handle);
  if (err == AEE_SUCCESS) s->backend_initialized = 0;
  return err;
}

extern "C" int htp_ops_session_create_channel(htp_ops_session *s, int fd, unsigned int max_msg_size) {
  if (!s || !s->handle) return -1;
  const int err = htp_ops_create_channel(s->handle, fd, max_msg_size);
  if (err == AEE_SUCCESS) s->channel_initialized = 1;
  return err;
}

extern "C" int htp_ops_session_create_channel_with_token(htp_ops_session *s, int fd, unsigned int max_msg_size) {
  if (!s || !s->handle) return -1;
  const int err = htp_ops_create_channel_with_token(s->handle, session_token(s), fd, max_msg_size);
  if (err == AEE_SUCCESS) s->channel_initialized = 1;
  return err;
}

extern "C" int htp_ops_session_destroy_channel(htp_ops_session *s) {
  if (!s || !s->handle) return -1;
  const int err = htp_ops_destroy_channel(s->handle);
  if (err == AEE_SUCCESS) s->channel_initialized = 0;
  return err;
}

extern "C" remote_handle64 htp_ops_session_handle(const htp_ops_session *s) {
  return s ? s->handle : static_cast<remote_handle64>(-1);
}

extern "C" int htp_ops_set_active_session(htp_ops_session *s) {
  if (!s || !s->handle) return -1;
  g_active_session = s;
  return 0;
}

extern "C" int htp_ops_set_default_session(void) {
  if (!g_default_session || !g_default_session->handle) return -1;
  g_active_session = g_default_session;
  return 0;
}

extern "C" uint32_t htp_ops_session_id(const htp_ops_session *s) { return s ? s->session_id : 0; }
extern "C" uint32_t htp_ops_session_domain(const htp_ops_session *s) { return s ? s->effective_domain_id : 0; }
extern "C" int htp_ops_session_is_reserved(const htp_ops_session *s) { return s && s->reserved; }
extern "C" int htp_ops_session_is_initialized(const htp_ops_session *s) { return s && s->backend_initialized; }
extern "C" int htp_ops_session_has_channel(const htp_ops_session *s) { return s && s->channel_initialized; }

extern "C" void htp_ops_session_close(htp_ops_session *s) {
  if (!s) return;
  if (s->handle) {
    if (s->channel_initialized) htp_ops_destroy_channel(s->handle);
    htp_ops_close(s->handle);
  }
  if (s->reserved && s->session_index < kMaxReserved) g_reserved_used[s->session_index] = 0;
  if (g_active_session == s) g_active_session = g_default_session == s ? nullptr : g_default_session;
  if (g_default_session == s) g_default_session = nullptr;
  delete s;
}

extern "C" remote_handle64 get_global_handle(void) {
  if (g_active_session) return g_active_session->handle;
  return g_default_session ? g_default_session->handle : static_cast<remote_handle64>(-1);
}

extern "C" int open_dsp_session(int domain_id, int unsigned_pd_enabled) {
  (void)unsigned_pd_enabled;
  if (g_default_session) return 0;
  const int err = htp_ops_session_open(&g_default_session, domain_id, nullptr, 0);
  if (err == 0) g_active_session = g_default_session;
  return err;
}

extern "C" void close_dsp_session(void) {
  htp_ops_session_close(g_default_session);
  g_default_session = nullptr;
  g_active_session = nullptr;
}

extern "C" void init_htp_backend(void) {
  if (g_default_session) (void)htp_ops_session_init_backend(g_default_session);
}

extern "C" int release_htp_backend(void) { return htp_ops_session_release_backend(g_default_session); }

extern "C" int create_htp_message_channel(int fd, unsigned int max_msg_size) {
  return htp_ops_session_create_channel(g_default_session, fd, max_msg_size);
}

extern "C" int destroy_htp_message_channel(void) { return htp_ops_session_destroy_channel(g_default_session); }

// ================================================================ op exports
extern "C" int htp_ops_rpc_rms_norm_f32(int dst_fd, int dst_offset, int src_fd, int src_offset, int ne0, int ne1) {
  return htp_ops_rms_norm_f32(get_global_handle(), dst_fd, dst_offset, src_fd, src_offset, ne0, ne1);
}
extern "C" int htp_ops_rpc_rms_norm_f32_session(htp_ops_session *s, int dst_fd, int dst_offset, int src_fd,
                                                int src_offset, int ne0, int ne1) {
  return htp_ops_rms_norm_f32(htp_ops_session_handle(s), dst_fd, dst_offset, src_fd, src_offset, ne0, ne1);
}
extern "C" int htp_ops_rpc_mat_mul_permuted_w16a32(int output_fd, int output_offset, int activation_fd,
                                                   int activation_offset, int weight_fd, int weight_offset,
                                                   int m, int k, int n) {
  return htp_ops_mat_mul_permuted_w16a32(get_global_handle(), output_fd, output_offset, activation_fd,
                                         activation_offset, weight_fd, weight_offset, m, k, n);
}
extern "C" int htp_ops_rpc_mat_mul_permuted_w16a32_session(htp_ops_session *s, int output_fd, int output_offset,
                                                           int activation_fd, int activation_offset,
                                                           int weight_fd, int weight_offset, int m, int k,
                                                           int n) {
  return htp_ops_mat_mul_permuted_w16a32(htp_ops_session_handle(s), output_fd, output_offset, activation_fd,
                                         activation_offset, weight_fd, weight_offset, m, k, n);
}
extern "C" int htp_ops_rpc_mat_mul_permuted_w16a32_trace_session(
    htp_ops_session *s, int output_fd, int output_offset, int activation_fd, int activation_offset,
    int weight_fd, int weight_offset, int m, int k, int n, uint64_t *activation_hash, uint64_t *output_hash,
    uint64_t *output_hash_after_remap) {
  return htp_ops_mat_mul_permuted_w16a32_trace(htp_ops_session_handle(s), output_fd, output_offset,
                                               activation_fd, activation_offset, weight_fd, weight_offset, m, k,
                                               n, activation_hash, output_hash, output_hash_after_remap);
}

extern "C" int htp_ops_f16_epilogue_version(void) { return 1; }
extern "C" int htp_ops_native_model_version(void) { return 0; }
extern "C" int htp_ops_dit_aux_version(void) { return 0; }
extern "C" int htp_ops_dit_concat_version(void) { return 0; }
extern "C" int htp_ops_w8a8_epilogue_version(void) { return 1; }
