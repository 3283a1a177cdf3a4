// Device-pointer C ABI of libhtp_ops_b200.so (include/htp_ops_b200.h): device
// context, TMA tensor maps, prepared-weight cache, workspace, plans, and the
// reference's kernel-level entry points (include/dsp/ops.h:20-31 of the
// reference) on top of them.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/htp_ops_b200.h"
#include "../../include/op_reg.h"
#include "kernels.h"
#include "scratch_run.h"

using namespace htpg;

// ------------------------------------------------------------------ state
namespace {

__device__ uint32_t g_watchdog;  // bits set by bounded device waits that expired

thread_local std::string t_last_cuda_error;
thread_local float t_phase_ms[3] = {0, 0, 0};
std::mutex g_mu;
int g_profiling = 0;

// benchmark phase timing: event triples recorded by runs, read back later
struct PhaseEvents {
  cudaEvent_t e[3];
};
bool g_phase_on = false;
std::vector<PhaseEvents> g_phase_pending, g_phase_free;

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Workspace {
  void *base = nullptr;
  size_t bytes = 0;
};

struct Device {
  bool ready = false;
  int ordinal = -1;
  int sms = 148;
  uint32_t *watchdog = nullptr;
  std::map<cudaStream_t, Workspace> ws;
  std::map<cudaStream_t, Workspace> qws;  // opcodes 2-4: counters | partials | FP16 operands
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
};

Device g_dev[16];
EncodeTiledFn g_encode = nullptr;

int record_cuda(cudaError_t e, int code = HTPG_ELAUNCH) {
  if (e == cudaSuccess) return HTPG_OK;
  t_last_cuda_error = cudaGetErrorString(e);
  if (std::getenv("HTPG_LOG")) std::fprintf(stderr, "htpg: CUDA error: %s\n", cudaGetErrorString(e));
  return code;
}

int current_device(Device **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return HTPG_ELAUNCH;
  Device &d = g_dev[dev];
  if (!d.ready) {
    const int rc = htpg_init(dev);
    if (rc != HTPG_OK) return rc;
  }
  *out = &d;
  return HTPG_OK;
}

// Zero every stream workspace of the device (W8A8/FP16 split-K areas and the
// opcode 2-4 stream-K scratch); the device is idle when this is called.
void clear_workspaces(Device *d) {
  for (auto *m : {&d->ws, &d->qws})
    for (auto &kv : *m)
      if (kv.second.base && cudaMemset(kv.second.base, 0, kv.second.bytes) != cudaSuccess) cudaGetLastError();
  cudaDeviceSynchronize();
  cudaGetLastError();
}

// NULL is the CUDA default stream (the stream torch and most callers use
// unless they create their own).
cudaStream_t pick_stream(Device *, void *stream) { return static_cast<cudaStream_t>(stream); }

// Stream-private scratch: activation codes / FP16 activations, row scales,
// split-K accumulators.  Grows (after a stream synchronisation) when a larger
// shape arrives; kept for the life of the library otherwise.
int workspace(Device *d, cudaStream_t st, size_t bytes, void **out) {
  Workspace &w = d->ws[st];
  if (w.bytes < bytes) {
    if (w.base) {
      cudaStreamSynchronize(st);
      cudaFree(w.base);
      w.base = nullptr;
      w.bytes = 0;
    }
    size_t want = bytes + bytes / 4 + (1u << 20);
    if (cudaMalloc(&w.base, want) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ENOMEM;
    }
    // split-K accumulators and counters must start (and are left) at zero
    if (cudaMemsetAsync(w.base, 0, want, st) != cudaSuccess) return HTPG_ELAUNCH;
    w.bytes = want;
  }
  *out = w.base;
  return HTPG_OK;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Largest split-K footprint: 128 weight tiles x 128 rows x 32 activation rows
// of INT32, plus one counter per tile.
constexpr size_t kSplitKRegion = 128u * 128u * 32u * 4u + 4096u;

// 2-D K-major tensor map: `rows` rows of `k` elements, row pitch `pitch`
// bytes, box = 128 bytes of K x box_rows rows, 128-byte swizzle, zero fill.
int make_map(CUtensorMap *map, const void *base, Kind kind, int k, int rows, size_t pitch,
             int box_rows) {
  if (!g_encode) return HTPG_ELAUNCH;
  const int esize = kind == Kind::I8 ? 1 : 2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esize), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, kind == Kind::I8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              2, const_cast<void *>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = "cuTensorMapEncodeTiled failed (" + std::to_string(static_cast<int>(r)) + ")";
    return HTPG_ELAUNCH;
  }
  return HTPG_OK;
}

// Row-major FP32 output [rows][cols] with row pitch ldo floats: 32 x 32 boxes,
// 128-byte swizzle (the epilogue's staging layout).
int make_out_map(CUtensorMap *map, float *out, int rows, int cols, long long ldo) {
  if (!g_encode) return HTPG_ELAUNCH;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldo) * 4u};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, out, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    t_last_cuda_error = "cuTensorMapEncodeTiled(out) failed (" + std::to_string(static_cast<int>(r)) + ")";
    return HTPG_ELAUNCH;
  }
  return HTPG_OK;
}

}  // namespace

// Prepared weight: K-major rows in HBM plus the per-column epilogue data.
struct htpg_weights {
  Kind kind = Kind::I8;
  int k = 0, ncols = 0, n0 = 0, n_total = 0;
  int device = 0;
  void *wk = nullptr;          // k-block-major [KB][ncols][128 B] int8 / fp16
  float *sw = nullptr;         // I8: [ncols] column scales
  int32_t *corr = nullptr;     // I8: [ncols] zero-point correction differences
  int32_t *sum7 = nullptr;     // I8: [ncols] (sum_k w) << 7, for the plane export
  float *inverse = nullptr;    // I8: [k], nullptr when every entry is 1.0
  int qtype = 0;               // QK0: ggml type; wk holds the stage records
  std::map<int, CUtensorMap> maps;  // by box rows
};

namespace {

int weight_map(htpg_weights *w, int box_rows, const CUtensorMap **out) {
  auto it = w->maps.find(box_rows);
  if (it == w->maps.end()) {
    CUtensorMap m;
    // rows kb * ncols + n of 128 bytes; a box is box_rows consecutive columns
    // of one k-block.  Boxes of a partial last column tile run into the next
    // k-block's rows: those columns are outside [0, ncols) and never stored.
    const int rows = kblocks(w->kind, w->k) * w->ncols;
    const int rc = make_map(&m, w->wk, w->kind, w->kind == Kind::I8 ? 128 : 64, rows, 128u, box_rows);
    if (rc != HTPG_OK) return rc;
    it = w->maps.emplace(box_rows, m).first;
  }
  *out = &it->second;
  return HTPG_OK;
}

// pointer-keyed cache of prepared weights for the one-call entry points
typedef std::tuple<const void *, int, int, int, int> CacheKey;  // ptr, kind, k, n, device
std::map<CacheKey, htpg_weights *> g_cache;


}  // namespace

// ================================================================ library
extern "C" int htpg_version(void) { return 1; }

extern "C" const char *htpg_strerror(int code) {
  switch (code) {
    case HTPG_OK: return "ok";
    case HTPG_EPAYLOAD: return "bad payload size or shape";
    case HTPG_EUNMAPPED: return "buffer not registered or too small";
    case HTPG_EHEADER: return "constants header or alignment mismatch";
    case HTPG_EARGS: return "null pointer or shape out of range";
    case HTPG_ECAPACITY: return "shape constraint violated";
    case HTPG_ECONTROL: return "alignment or control block error";
    case HTPG_ELAUNCH: return "CUDA launch or stream error";
    case HTPG_ENOPLAN: return "no tile plan for this shape";
    case HTPG_EWATCHDOG: return "device wait expired";
    case HTPG_ENOMEM: return "device allocation failed";
    case HTPG_ESCRATCH: return "request does not fit the static scratch array";
    case HTPG_EARCH: return "device is not sm_100";
    default: return "unknown error";
  }
}

extern "C" const char *htpg_last_cuda_error(void) { return t_last_cuda_error.c_str(); }

extern "C" int htpg_init(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (device < 0 || device >= 16) return HTPG_EARGS;
  Device &d = g_dev[device];
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return HTPG_ELAUNCH;
  }
  if (d.ready) return HTPG_OK;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return record_cuda(cudaGetLastError());
  if (prop.major != 10 || prop.minor != 0) return HTPG_EARCH;
  if (!g_encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return record_cuda(cudaErrorNotSupported);
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
  d.ordinal = device;
  d.sms = prop.multiProcessorCount;
  if (cudaGetSymbolAddress(reinterpret_cast<void **>(&d.watchdog), g_watchdog) != cudaSuccess)
    return record_cuda(cudaGetLastError());
  for (auto &e : d.ev)
    if (cudaEventCreate(&e) != cudaSuccess) return record_cuda(cudaGetLastError());
  d.ready = true;
  return HTPG_OK;
}

extern "C" int htpg_check_device(void *stream, uint32_t *flags) {
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t st = pick_stream(d, stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return record_cuda(cudaGetLastError());
  uint32_t v = 0;
  if (cudaMemcpyFromSymbol(&v, g_watchdog, sizeof(v)) != cudaSuccess) return record_cuda(cudaGetLastError());
  if (v) {
    const uint32_t zero = 0;
    cudaMemcpyToSymbol(g_watchdog, &zero, sizeof(zero));
    // A launch that gave up may have left split-K partial sums and arrival
    // counters behind, in the W8A8/FP16 workspaces and in the opcode 2-4
    // stream-K scratch alike; both rely on "left zero by every launch".
    // Other streams of this device may still run: wait for them first.
    cudaDeviceSynchronize();
    cudaGetLastError();
    clear_workspaces(d);
  }
  if (flags) *flags = v;
  return v ? HTPG_EWATCHDOG : HTPG_OK;
}

// Test hook: leave the state an aborted launch can leave (every stream
// workspace of the current device filled with `fill`, the split-K watchdog
// bit set), so a test can check that htpg_check_device restores it.
extern "C" int htpg_debug_simulate_abort(uint32_t fill) {
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  if (cudaDeviceSynchronize() != cudaSuccess) return record_cuda(cudaGetLastError());
  for (auto *m : {&d->ws, &d->qws})
    for (auto &kv : *m)
      if (kv.second.base && cudaMemset(kv.second.base, static_cast<int>(fill & 0xffu), kv.second.bytes) != cudaSuccess)
        return record_cuda(cudaGetLastError());
  const uint32_t bit = 8u;  // the split-K role bit of the watchdog word
  if (cudaMemcpyToSymbol(g_watchdog, &bit, sizeof(bit)) != cudaSuccess) return record_cuda(cudaGetLastError());
  return HTPG_OK;
}

extern "C" int htpg_debug_workspaces(size_t *ws_bytes, size_t *qws_bytes) {
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  size_t a = 0, b = 0;
  for (auto &kv : d->ws) a += kv.second.bytes;
  for (auto &kv : d->qws) b += kv.second.bytes;
  if (ws_bytes) *ws_bytes = a;
  if (qws_bytes) *qws_bytes = b;
  return HTPG_OK;
}

extern "C" uint64_t htpg_launch_count(void) { return htpg::launches(); }

extern "C" int htpg_phase_timing(int on) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_phase_on = on != 0;
  return HTPG_OK;
}

extern "C" int htpg_phase_timing_read(double *act_ms, double *gemm_ms, int *runs) {
  std::lock_guard<std::mutex> lk(g_mu);
  double a = 0, g = 0;
  int n = 0;
  for (auto &pe : g_phase_pending) {
    float t01 = 0, t12 = 0;
    if (cudaEventSynchronize(pe.e[2]) != cudaSuccess) return record_cuda(cudaGetLastError());
    cudaEventElapsedTime(&t01, pe.e[0], pe.e[1]);
    cudaEventElapsedTime(&t12, pe.e[1], pe.e[2]);
    a += t01;
    g += t12;
    ++n;
    g_phase_free.push_back(pe);
  }
  g_phase_pending.clear();
  if (act_ms) *act_ms = a;
  if (gemm_ms) *gemm_ms = g;
  if (runs) *runs = n;
  return HTPG_OK;
}

extern "C" int htpg_plan_info(int kind, int m, int n, int k, int sms, int64_t out[12]) {
  if (!out || m < 1 || n < 1 || k < 1 || sms < 1 || (kind != 0 && kind != 1)) return HTPG_EARGS;
  const GemmPlan p = plan_for(kind == 0 ? Kind::I8 : Kind::F16, m, n, k, sms, 0, 1);
  const int64_t v[12] = {p.reg ? 2 : p.swap ? 1 : p.pair_sw ? 3 : 0,
                         p.bn,
                         p.splits,
                         p.tiles_a,
                         p.tiles_b,
                         p.kb_total,
                         p.kb_per_split,
                         p.units,
                         p.grid,
                         static_cast<int64_t>(p.smem),
                         p.tail_s > 1 ? p.full_units : p.units,
                         p.tail_s};
  for (int i = 0; i < 12; ++i) out[i] = v[i];
  return HTPG_OK;
}

extern "C" int htpg_stream_read(const void *src, size_t bytes, void *stream) {
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  if (!src || !bytes || bytes % 32 || (reinterpret_cast<uintptr_t>(src) & 31u)) return HTPG_EARGS;
  return record_cuda(launch_stream_read(src, bytes, d->sms, pick_stream(d, stream)));
}

extern "C" int htpg_set_qk0_decode(int which) {
  if (which < 0 || which > 2) return HTPG_EARGS;
  g_qdec.store(which == 0 ? 1 : which == 1 ? 0 : 2);
  return HTPG_OK;
}

extern "C" int htpg_set_qdec_shape(int per_sm, int tiles) {
  if (per_sm == 0 && tiles == 0) {
    g_qdec_shape.store(0);
    return HTPG_OK;
  }
  if ((per_sm != 1 && per_sm != 2) || (tiles != 16 && tiles != 8 && tiles != 4)) return HTPG_EARGS;
  g_qdec_shape.store(per_sm * 100 + tiles);
  return HTPG_OK;
}

extern "C" int htpg_set_pair_tail_split(int on) {
  if (on != 0 && on != 1) return HTPG_EARGS;
  g_pair_tail.store(on);
  return HTPG_OK;
}

extern "C" int htpg_set_pair_direct(int on) {
  if (on != 0 && on != 1) return HTPG_EARGS;
  g_pair_direct.store(on);
  return HTPG_OK;
}


extern "C" int htpg_set_decode_kernel(int which) {
  if (which != 0 && which != 1) return HTPG_EARGS;
  g_decode_kernel.store(which);
  return HTPG_OK;
}

extern "C" int htpg_set_profiling(int on) {
  g_profiling = on ? 1 : 0;
  return HTPG_OK;
}

extern "C" int htpg_last_phase_ms(float *quant_ms, float *gemm_ms, float *total_ms) {
  if (quant_ms) *quant_ms = t_phase_ms[0];
  if (gemm_ms) *gemm_ms = t_phase_ms[1];
  if (total_ms) *total_ms = t_phase_ms[2];
  return HTPG_OK;
}

// ================================================================ quantise
extern "C" int htpg_quantize_rows(int8_t *codes, float *row_scales, const float *x,
                                  const float *inverse, int m, int k, void *stream) {
  if (!codes || !row_scales || !x || m < 1 || k < 32 || k % 32) return HTPG_EARGS;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(codes)) & 15u) return HTPG_ECONTROL;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  return record_cuda(launch_quantize_rows(codes, row_scales, x, inverse, m, k, pick_stream(d, stream)));
}

// ================================================================ weights
extern "C" int htpg_weights_cols(const htpg_weights *w) { return w ? w->ncols : 0; }

extern "C" void htpg_weights_destroy(htpg_weights *w) {
  if (!w) return;
  cudaFree(w->wk);
  cudaFree(w->sw);
  cudaFree(w->corr);
  cudaFree(w->sum7);
  cudaFree(w->inverse);
  delete w;
}

extern "C" int htpg_w8a8_weights_create(const void *constants, int k, int n, int n0, int n_cols,
                                        void *stream, htpg_weights **out) {
  if (!out) return HTPG_EARGS;
  *out = nullptr;
  if (!constants || k < 32 || k > HTPG_W8A8_MAX_K || n < 64 || n > HTPG_W8A8_MAX_N) return HTPG_EARGS;
  if (k % 32 || n % 64) return HTPG_ECAPACITY;
  if (n_cols == 0) n_cols = n - n0;
  if (n0 < 0 || n0 % 64 || n_cols < 64 || n_cols % 64 || n0 + n_cols > n) return HTPG_ECAPACITY;
  if (reinterpret_cast<uintptr_t>(constants) & 15u) return HTPG_ECONTROL;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t st = pick_stream(d, stream);
  W8A8Header h;
  if (cudaMemcpyAsync(&h, constants, sizeof(h), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return record_cuda(cudaGetLastError());
  const size_t kn = static_cast<size_t>(k) * n;
  const size_t bytes = 128u + kn + 8u * n + 4u * static_cast<size_t>(k);
  // same acceptance rules as the reference executor (op_executor.cc:331-335)
  if (h.magic != W8A8_HEADER_MAGIC || h.version != W8A8_HEADER_VERSION || h.k != static_cast<uint32_t>(k) ||
      h.n != static_cast<uint32_t>(n) || h.weight_offset != 128 || h.scale_offset != 128u + kn ||
      h.sum_offset != h.scale_offset + 4u * n || h.inverse_offset != h.sum_offset + 4u * n ||
      h.bytes != bytes)
    return HTPG_EHEADER;
  const uint8_t *blob = static_cast<const uint8_t *>(constants);
  htpg_weights *w = new htpg_weights;
  w->kind = Kind::I8;
  w->k = k;
  w->ncols = n_cols;
  w->n0 = n0;
  w->n_total = n;
  w->device = d->ordinal;
  uint32_t *flag = nullptr;
  const size_t wk_bytes = kblock_bytes(Kind::I8, k, n_cols);
  bool ok = cudaMalloc(&w->wk, wk_bytes) == cudaSuccess &&
            cudaMalloc(&w->sw, 4u * n_cols) == cudaSuccess &&
            cudaMalloc(&w->corr, 4u * n_cols) == cudaSuccess && cudaMalloc(&w->sum7, 4u * n_cols) == cudaSuccess &&
            cudaMalloc(&w->inverse, 4u * k) == cudaSuccess && cudaMalloc(&flag, 4) == cudaSuccess;
  if (!ok) {
    cudaGetLastError();
    cudaFree(flag);
    htpg_weights_destroy(w);
    return HTPG_ENOMEM;
  }
  // the zero padding of a partial last k-block adds nothing to the products
  cudaError_t e = k % 128 ? cudaMemsetAsync(w->wk, 0, wk_bytes, st) : cudaSuccess;
  if (e == cudaSuccess)
    e = launch_repack_w8(static_cast<int8_t *>(w->wk), blob + h.weight_offset, k, n0, n_cols, st);
  if (e == cudaSuccess)
    e = launch_colsum_corr(w->corr, w->sum7, static_cast<const int8_t *>(w->wk),
                           reinterpret_cast<const int32_t *>(blob + h.sum_offset), k, n0, n_cols, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(w->sw, blob + h.scale_offset + 4u * n0, 4u * n_cols, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(w->inverse, blob + h.inverse_offset, 4u * k, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(flag, 0, 4, st);
  if (e == cudaSuccess) e = launch_check_ones(flag, w->inverse, k, st);
  uint32_t not_ones = 1;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&not_ones, flag, 4, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  cudaFree(flag);
  if (e != cudaSuccess) {
    htpg_weights_destroy(w);
    return record_cuda(e);
  }
  if (!not_ones) {  // x*1.0f == x exactly: skip the multiply
    cudaFree(w->inverse);
    w->inverse = nullptr;
  }
  *out = w;
  return HTPG_OK;
}

extern "C" int htpg_f16_weights_create(const uint16_t *permuted_weight, int k, int n, int n0,
                                       int n_cols, void *stream, htpg_weights **out) {
  if (!out) return HTPG_EARGS;
  *out = nullptr;
  if (!permuted_weight || k < 32 || n < 32) return HTPG_EARGS;
  if (k % 32 || n % 32) return HTPG_ECAPACITY;
  if (n_cols == 0) n_cols = n - n0;
  if (n0 < 0 || n0 % 32 || n_cols < 32 || n_cols % 32 || n0 + n_cols > n) return HTPG_ECAPACITY;
  if (reinterpret_cast<uintptr_t>(permuted_weight) & 3u) return HTPG_ECONTROL;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t st = pick_stream(d, stream);
  htpg_weights *w = new htpg_weights;
  w->kind = Kind::F16;
  w->k = k;
  w->ncols = n_cols;
  w->n0 = n0;
  w->n_total = n;
  w->device = d->ordinal;
  const size_t wk_bytes = kblock_bytes(Kind::F16, k, n_cols);
  if (cudaMalloc(&w->wk, wk_bytes) != cudaSuccess) {
    cudaGetLastError();
    delete w;
    return HTPG_ENOMEM;
  }
  cudaError_t e = k % 64 ? cudaMemsetAsync(w->wk, 0, wk_bytes, st) : cudaSuccess;
  if (e == cudaSuccess)
    e = launch_repack_f16(static_cast<uint16_t *>(w->wk), permuted_weight, k, n0, n_cols, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    htpg_weights_destroy(w);
    return record_cuda(e);
  }
  *out = w;
  return HTPG_OK;
}

// ================================================================ run
namespace {

// outs[0..n_outs): destinations of the output (n_outs > 1: the same output
// block in several buffers, each written by TMA stores from the epilogue).
// act_f16: FP16 activations [m][k] already in HBM (FP16 weights only; x is
// then unused and no conversion runs).
int run_common(htpg_weights *w, float *const *outs, int n_outs, int ldo, const float *x,
               const float *bias, int m, int channels, int mode, void *stream,
               const float **row_scales_out = nullptr, const uint16_t *act_f16 = nullptr,
               bool late_weights = false) {
  if (act_f16 && w && w->kind != Kind::F16) return HTPG_EARGS;
  if (w && w->kind == Kind::QK0) return HTPG_EARGS;
  if (!w || !outs || n_outs < 1 || n_outs > kMaxOutputs || (!x && !act_f16)) return HTPG_EARGS;
  for (int i = 0; i < n_outs; ++i)
    if (!outs[i]) return HTPG_EARGS;
  float *out = outs[0];
  const int n = w->ncols, k = w->k;
  if (m < 1 || m > HTPG_W8A8_MAX_M) return HTPG_EARGS;
  if (mode < 0 || mode > HTPG_MODE_PLANES || (mode == HTPG_MODE_PLANES && w->kind != Kind::I8))
    return HTPG_ECAPACITY;
  if (channels == 0) channels = n;
  if (channels < 1 || channels > n || (mode != 3 && channels != n)) return HTPG_ECAPACITY;
  if ((reinterpret_cast<uintptr_t>(act_f16 ? static_cast<const void *>(act_f16) : x)) & 15u) return HTPG_ECONTROL;
  if (reinterpret_cast<uintptr_t>(out) & 3u) return HTPG_ECONTROL;
  if (ldo == 0) ldo = mode == 3 ? m : n;
  if ((mode == 3 && ldo < m) || (mode != 3 && ldo < n) || (mode == HTPG_MODE_PLANES && ldo != n))
    return HTPG_EARGS;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t st = pick_stream(d, stream);
  std::lock_guard<std::mutex> lk(g_mu);

  const GemmPlan plan = plan_for(w->kind, m, n, k, d->sms, mode, n_outs);
  // several destinations need the TMA-store epilogue (normal orientation, row-major, aligned)
  if (n_outs > 1 && (plan.swap || plan.pair_sw || mode == 3 || !tma_store_ok(out, ldo))) return HTPG_ECAPACITY;
  // the weight is the A operand of swapped plans (small M and swapped CTA pairs)
  const bool w_is_a = plan.swap || plan.pair_sw;
  // Workspace: [split-K accumulators + counters | activation codes / FP16 | row scales].
  // The split-K region sits at a fixed offset and is kept all-zero (zeroed at
  // allocation, left zeroed by every launch), so no per-call clear is needed.
  const size_t wsk_bytes = kSplitKRegion;
  if (splitk_ws_bytes(plan) + splitk_count_bytes(plan) > wsk_bytes) return HTPG_ENOPLAN;
  const size_t act_elem = w->kind == Kind::I8 ? 1 : 2;
  const size_t act_bytes = act_f16 ? 0 : align_up(static_cast<size_t>(m) * k * act_elem, 1024);
  const size_t scale_bytes = align_up(4u * static_cast<size_t>(m), 1024);
  // the tail pieces' INT32 sums (written before they are read: no clearing)
  const size_t slot_bytes = tail_slot_bytes(plan);
  void *base = nullptr;
  rc = workspace(d, st, wsk_bytes + act_bytes + scale_bytes + slot_bytes, &base);
  if (rc) return rc;
  int32_t *wsk = slot_bytes ? reinterpret_cast<int32_t *>(static_cast<uint8_t *>(base) + wsk_bytes + act_bytes +
                                                          scale_bytes)
                            : static_cast<int32_t *>(base);
  uint32_t *cnt = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(base) + splitk_ws_bytes(plan));
  uint8_t *act = act_f16 ? reinterpret_cast<uint8_t *>(const_cast<uint16_t *>(act_f16))
                         : static_cast<uint8_t *>(base) + wsk_bytes;
  float *scales = reinterpret_cast<float *>(static_cast<uint8_t *>(base) + wsk_bytes + act_bytes);
  if (row_scales_out) *row_scales_out = scales;

  const bool prof = g_profiling != 0;
  PhaseEvents pe;
  const bool phase = g_phase_on;
  if (phase) {
    if (g_phase_free.empty()) {
      for (auto &e : pe.e) cudaEventCreate(&e);
    } else {
      pe = g_phase_free.back();
      g_phase_free.pop_back();
    }
    cudaEventRecord(pe.e[0], st);
  }
  if (prof) cudaEventRecord(d->ev[0], st);
  cudaError_t e = cudaSuccess;
  if (w->kind == Kind::I8)
    e = launch_quantize_rows(reinterpret_cast<int8_t *>(act), scales, x, w->inverse, m, k, st);
  else if (!act_f16)
    e = launch_to_f16(reinterpret_cast<uint16_t *>(act), x, static_cast<long long>(m) * k, st);
  if (e != cudaSuccess) return record_cuda(e);
  if (prof) cudaEventRecord(d->ev[1], st);
  if (phase) cudaEventRecord(pe.e[1], st);

  CUtensorMap act_map;
  const CUtensorMap *wmap = nullptr;
  rc = make_map(&act_map, act, w->kind, k, m, static_cast<size_t>(k) * act_elem,
                plan.pair_sw ? plan.bn / 2 : plan.swap ? plan.bn : 128);
  if (rc) return rc;
  rc = weight_map(w, w_is_a ? 128 : box_rows_b(plan), &wmap);
  if (rc) return rc;

  GemmArgs a;
  a.M = m;
  a.N = n;
  a.K = k;
  a.out = out;
  a.ldo = ldo;
  a.mode = mode;
  a.channels = channels;
  a.row_scale = scales;
  a.col_scale = w->sw;
  a.col_corr = w->corr;
  a.col_sum7 = w->sum7;
  a.bias = bias;
  a.ws = wsk;
  a.ws_count = cnt;
  a.watchdog = d->watchdog;
  a.wk = w->wk;
  a.act = act;
  a.late_weights = late_weights ? 1 : 0;
  // row-major outputs of the normal orientation leave the SM through TMA stores
  OutMaps out_maps;
  if (mode == HTPG_MODE_PLANES) {
    a.tma_store = tma_store_ok(out, ldo) ? 1 : 0;  // 16-byte aligned rows: vector plane stores
  } else if (!w_is_a && mode != 3 && tma_store_ok(out, ldo)) {
    for (int i = 0; i < n_outs; ++i) {
      if (!tma_store_ok(outs[i], ldo)) return HTPG_ECONTROL;
      rc = make_out_map(&out_maps.map[i], outs[i], m, n, ldo);
      if (rc) return rc;
    }
    out_maps.count = n_outs;
    a.tma_store = 1;
  }
  e = w_is_a ? launch_gemm(plan, *wmap, act_map, out_maps, a, st)
             : launch_gemm(plan, act_map, *wmap, out_maps, a, st);
  if (e != cudaSuccess) return record_cuda(e);
  if (phase) {
    cudaEventRecord(pe.e[2], st);
    g_phase_pending.push_back(pe);
  }
  if (prof) {
    cudaEventRecord(d->ev[2], st);
    cudaEventSynchronize(d->ev[2]);
    cudaEventElapsedTime(&t_phase_ms[0], d->ev[0], d->ev[1]);
    cudaEventElapsedTime(&t_phase_ms[1], d->ev[1], d->ev[2]);
    cudaEventElapsedTime(&t_phase_ms[2], d->ev[0], d->ev[2]);
  }
  return HTPG_OK;
}

}  // namespace

extern "C" int htpg_w8a8_run(const htpg_weights *w, float *out, int ldo, const float *x,
                             const float *bias, int m, int channels, int mode, void *stream) {
  if (!w || w->kind != Kind::I8) return HTPG_EARGS;
  return run_common(const_cast<htpg_weights *>(w), &out, 1, ldo, x, bias, m, channels, mode, stream);
}

extern "C" int htpg_f16_run(const htpg_weights *w, float *out, int ldo, const float *x,
                            const float *bias, int m, int channels, int mode, void *stream) {
  if (!w || w->kind != Kind::F16) return HTPG_EARGS;
  return run_common(const_cast<htpg_weights *>(w), &out, 1, ldo, x, bias, m, channels, mode, stream);
}

namespace {
// Control block of the CPU-epilogue form, filled after the planes are written
// (linear_w8a8.c:421-427, 512-526).  This build computes all M rows in one
// batch and streams the weight once; it has no VTCM (vtcm_bytes 0).
int fill_control(W8A8CpuControl *control, const float *scales_dev, int m, int k, int n, cudaStream_t st) {
  cudaError_t e = cudaMemcpyAsync(control->scales, scales_dev, 4u * static_cast<size_t>(m),
                                  cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return record_cuda(e);
  control->vtcm_bytes = 0;
  control->activation_rows = static_cast<uint32_t>(m);
  control->weight_columns = static_cast<uint32_t>(n / 64);
  control->weight_loads = 1;
  control->weight_loaded_bytes = static_cast<uint64_t>(k) * static_cast<uint64_t>(n);
  control->batches[0].m0 = 0;
  control->batches[0].rows = m;
  control->batches[0].n0 = 0;
  control->batches[0].columns = n / 64;
  std::atomic_thread_fence(std::memory_order_release);
  reinterpret_cast<volatile uint32_t *>(&control->produced)[0] = 1u;  // published last
  return HTPG_OK;
}
}  // namespace

extern "C" int htpg_w8a8_run_planes(const htpg_weights *w, float *dst, const float *x, int m,
                                    struct W8A8CpuControl *control, void *stream) {
  if (!control) return HTPG_ECONTROL;
  if (!w || w->kind != Kind::I8 || !dst || !x) return HTPG_EARGS;
  if (m < 1 || m > 4096) return HTPG_EARGS;  // the control block holds 4096 row scales
  const float *scales = nullptr;
  float *outs[1] = {dst};
  int rc = run_common(const_cast<htpg_weights *>(w), outs, 1, 0, x, nullptr, m, 0, HTPG_MODE_PLANES, stream,
                      &scales);
  if (rc) return rc;
  rc = htpg_check_device(stream, nullptr);
  if (rc) return rc;
  return fill_control(control, scales, m, w->k, w->ncols, static_cast<cudaStream_t>(stream));
}

extern "C" int htpg_w8a8_run_gather(const htpg_weights *w, float *const *outs, int n_outs, int ldo,
                                    const float *x, const float *bias, int m, int channels, int mode,
                                    void *stream) {
  if (!w || w->kind != Kind::I8) return HTPG_EARGS;
  return run_common(const_cast<htpg_weights *>(w), outs, n_outs, ldo, x, bias, m, channels, mode, stream);
}

// ---------------------------------------------------------------- opcode 17
namespace {
int cached_weights(Kind kind, const void *ptr, int k, int n, void *stream, htpg_weights **out, int qtype = 0);
// im2col staging, per device, grown as needed (one chunk of output rows)
struct ConvBuf {
  void *base = nullptr;
  size_t bytes = 0;
};
ConvBuf g_conv_buf[16];
size_t g_conv_chunk_bytes = 256u << 20;  // FP16 im2col bytes per GEMM launch (staging budget)

int conv_geometry_ok(const NativeConvParams *p) {
  // the executor's acceptance rules (op_executor.cc:405-418)
  if (p->iw <= 0 || p->ih <= 0 || p->ic <= 0 || p->oc <= 0 || p->batch <= 0 || p->ow <= 0 || p->oh <= 0 ||
      p->kw <= 0 || p->kh <= 0 || p->sx <= 0 || p->sy <= 0 || p->dx <= 0 || p->dy <= 0 || p->kp % 32 ||
      p->np % 32 || p->np < p->oc || p->kp < static_cast<int64_t>(p->kw) * p->kh * p->ic ||
      (p->upscale != 1 && p->upscale != 2) ||
      p->ow != (p->upscale * p->iw + 2 * p->px - p->dx * (p->kw - 1) - 1) / p->sx + 1 ||
      p->oh != (p->upscale * p->ih + 2 * p->py - p->dy * (p->kh - 1) - 1) / p->sy + 1)
    return 0;
  const size_t in_size = static_cast<size_t>(p->iw) * p->ih * p->ic * p->batch * 4;
  const size_t out_size = static_cast<size_t>(p->ow) * p->oh * p->oc * p->batch * 4;
  return in_size <= INT32_MAX && out_size <= INT32_MAX && static_cast<size_t>(p->kp) * p->np * 2 <= INT32_MAX;
}

// Per image: im2col of a chunk of output rows into FP16, then the FP16 GEMM
// (K = kp, N = np) with the bias + channel-major epilogue over oc channels
// (mat_mul.c:2291-2343).  times (optional, synchronises): gather and GEMM ms.
int conv_core(htpg_weights *w, float *dst, const float *x, const float *bias, const NativeConvParams *p,
              cudaStream_t st, double *gather_ms, double *gemm_ms) {
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  const int spatial = p->ow * p->oh;
  const size_t row_bytes = static_cast<size_t>(p->kp) * 2;
  int chunk = static_cast<int>(std::min<size_t>(spatial, std::max<size_t>(128, g_conv_chunk_bytes / row_bytes)));
  ConvBuf &cb = g_conv_buf[d->ordinal];
  const size_t need = static_cast<size_t>(chunk) * row_bytes;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cb.bytes < need) {
      if (cb.base) {
        cudaStreamSynchronize(st);
        cudaFree(cb.base);
        cb.base = nullptr;
        cb.bytes = 0;
      }
      if (cudaMalloc(&cb.base, need) != cudaSuccess) {
        cudaGetLastError();
        return HTPG_ENOMEM;
      }
      cb.bytes = need;
    }
  }
  const ConvGeom g = {p->iw, p->ih, p->ic, p->ow, p->oh, p->kw, p->kh, p->sx, p->sy,
                      p->px, p->py, p->dx, p->dy, p->kp, p->upscale};
  cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
  const bool timed = gather_ms || gemm_ms;
  if (timed) {
    for (auto &e : ev) cudaEventCreate(&e);
    *gather_ms = *gemm_ms = 0.0;
  }
  uint16_t *a = static_cast<uint16_t *>(cb.base);
  for (int b = 0; b < p->batch && rc == HTPG_OK; ++b) {
    const float *xb = x + static_cast<size_t>(b) * p->ic * p->ih * p->iw;
    for (int m0 = 0; m0 < spatial; m0 += chunk) {
      const int rows = std::min(chunk, spatial - m0);
      if (timed) cudaEventRecord(ev[0], st);
      cudaError_t e = launch_im2col_f16(a, xb, g, m0, rows, st);
      if (e != cudaSuccess) {
        rc = record_cuda(e);
        break;
      }
      if (timed) cudaEventRecord(ev[1], st);
      float *out = dst + static_cast<size_t>(b) * p->oc * spatial + m0;
      rc = run_common(w, &out, 1, spatial, nullptr, bias, rows, p->oc, 3, st, nullptr, a);
      if (rc) break;
      if (timed) {
        cudaEventRecord(ev[2], st);
        cudaEventSynchronize(ev[2]);
        float t01 = 0, t12 = 0;
        cudaEventElapsedTime(&t01, ev[0], ev[1]);
        cudaEventElapsedTime(&t12, ev[1], ev[2]);
        *gather_ms += t01;
        *gemm_ms += t12;
      }
    }
  }
  if (timed)
    for (auto &e : ev) cudaEventDestroy(e);
  return rc;
}
}  // namespace

extern "C" int htpg_conv_set_chunk_bytes(size_t bytes) {
  if (bytes == 0) return HTPG_EARGS;
  std::lock_guard<std::mutex> lk(g_mu);
  g_conv_chunk_bytes = bytes;
  return HTPG_OK;
}

extern "C" int htpg_conv2d_run(const htpg_weights *w, float *dst, const float *x, const float *bias,
                               const struct NativeConvParams *p, void *stream) {
  if (!w || w->kind != Kind::F16 || !dst || !x || !p) return HTPG_EARGS;
  if (!conv_geometry_ok(p)) return HTPG_EPAYLOAD;
  if (w->k != p->kp || w->ncols != p->np) return HTPG_EARGS;
  return conv_core(const_cast<htpg_weights *>(w), dst, x, bias, p, static_cast<cudaStream_t>(stream), nullptr,
                   nullptr);
}

extern "C" int hmx_conv2d_nchw_f16(float *dst, const float *input, const uint16_t *weight, const float *bias,
                                   struct NativeConvParams *p) {
  if (!dst || !input || !weight || !p) return HTPG_EARGS;
  if (!conv_geometry_ok(p)) return HTPG_EPAYLOAD;
  const auto t0 = std::chrono::steady_clock::now();
  htpg_weights *w = nullptr;
  int rc = cached_weights(Kind::F16, weight, p->kp, p->np, nullptr, &w);
  if (rc) return rc;
  const double weight_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  double gather_ms = 0, gemm_ms = 0;
  rc = conv_core(w, dst, input, bias, p, nullptr, &gather_ms, &gemm_ms);
  if (rc == HTPG_OK) rc = htpg_check_device(nullptr, nullptr);
  // the reference reports its phases in microseconds (mat_mul.c:2340); the
  // epilogue is fused into the GEMM here, so the store phase is 0
  p->gather_us = static_cast<int32_t>(gather_ms * 1e3);
  p->weight_us = static_cast<int32_t>(weight_ms * 1e3);
  p->hmx_us = static_cast<int32_t>(gemm_ms * 1e3);
  p->store_us = 0;
  return rc;
}

// ---------------------------------------------------------------- IPC
namespace {
typedef CUresult (*AddressRangeFn)(CUdeviceptr *, size_t *, CUdeviceptr);
std::map<void *, void *> g_ipc_bases;  // imported address -> base returned by the open
}  // namespace

extern "C" int htpg_ipc_export(const void *dev_ptr, void *handle) {
  if (!dev_ptr || !handle) return HTPG_EARGS;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  static AddressRangeFn range = nullptr;
  if (!range) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return record_cuda(cudaErrorNotSupported);
    range = reinterpret_cast<AddressRangeFn>(fn);
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return HTPG_EARGS;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) return record_cuda(e);
  const int64_t offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  std::memcpy(handle, &h, sizeof(h));
  std::memcpy(static_cast<uint8_t *>(handle) + sizeof(h), &offset, sizeof(offset));
  return HTPG_OK;
}

extern "C" int htpg_ipc_import(const void *handle, void **dev_ptr) {
  if (!handle || !dev_ptr) return HTPG_EARGS;
  *dev_ptr = nullptr;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  int64_t offset = 0;
  std::memcpy(&h, handle, sizeof(h));
  std::memcpy(&offset, static_cast<const uint8_t *>(handle) + sizeof(h), sizeof(offset));
  void *base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return record_cuda(e);
  void *p = static_cast<uint8_t *>(base) + offset;
  std::lock_guard<std::mutex> lk(g_mu);
  g_ipc_bases[p] = base;
  *dev_ptr = p;
  return HTPG_OK;
}

extern "C" int htpg_ipc_close(void *dev_ptr) {
  void *base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_ipc_bases.find(dev_ptr);
    if (it == g_ipc_bases.end()) return HTPG_EARGS;
    base = it->second;
    g_ipc_bases.erase(it);
  }
  return record_cuda(cudaIpcCloseMemHandle(base));
}

// W8A8 run whose scratch is the caller's fixed array [scratch, scratch+bytes)
// instead of the per-stream workspace: the allocation-free entry point
// (noalloc.cu) calls this.  Same checks and kernels as htpg_w8a8_run; no
// profiling or phase events.
int htpg::w8a8_run_in_scratch(const htpg_weights *w, float *out, int ldo, const float *x,
                              const float *bias, int m, int channels, int mode, void *stream,
                              void *scratch, size_t scratch_bytes) {
  if (!w || w->kind != Kind::I8 || !out || !x || !scratch) return HTPG_EARGS;
  const int n = w->ncols, k = w->k;
  if (m < 1 || m > HTPG_W8A8_MAX_M) return HTPG_EARGS;
  if (mode < 0 || mode > HTPG_MODE_RAW) return HTPG_ECAPACITY;
  if (channels == 0) channels = n;
  if (channels < 1 || channels > n || (mode != 3 && channels != n)) return HTPG_ECAPACITY;
  if (reinterpret_cast<uintptr_t>(x) & 15u) return HTPG_ECONTROL;
  if (reinterpret_cast<uintptr_t>(out) & 3u) return HTPG_ECONTROL;
  if (ldo == 0) ldo = mode == 3 ? m : n;
  if ((mode == 3 && ldo < m) || (mode != 3 && ldo < n)) return HTPG_EARGS;
  static_assert(kSplitKRegion == kStaticSplitKBytes, "split-K area size is part of the documented layout");
  const size_t act_bytes = align_up(static_cast<size_t>(m) * k, 1024);
  const size_t scale_bytes = align_up(4u * static_cast<size_t>(m), 1024);
  if (kSplitKRegion + act_bytes + scale_bytes > scratch_bytes) {
    t_last_cuda_error = "static scratch: m*k = " + std::to_string(static_cast<size_t>(m) * k) +
                        " needs " + std::to_string(kSplitKRegion + act_bytes + scale_bytes) +
                        " bytes, the array holds " + std::to_string(scratch_bytes);
    return HTPG_ESCRATCH;
  }
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t st = pick_stream(d, stream);
  std::lock_guard<std::mutex> lk(g_mu);

  // the documented scratch layout has no room for tail-piece sums: whole tiles only
  const GemmPlan plan = plan_for(Kind::I8, m, n, k, d->sms, mode, 1, false);
  const bool w_is_a = plan.swap || plan.pair_sw;
  const size_t splitk_bytes = splitk_ws_bytes(plan) + splitk_count_bytes(plan);
  if (splitk_bytes > kSplitKRegion) return HTPG_ENOPLAN;
  uint8_t *base = static_cast<uint8_t *>(scratch);
  int32_t *wsk = reinterpret_cast<int32_t *>(base);
  uint32_t *cnt = reinterpret_cast<uint32_t *>(base + splitk_ws_bytes(plan));
  int8_t *act = reinterpret_cast<int8_t *>(base + kSplitKRegion);
  float *scales = reinterpret_cast<float *>(base + kSplitKRegion + act_bytes);
  // The array keeps whatever the previous call (or an aborted launch) left:
  // the split-K partial sums and tile counters must start at zero.
  cudaError_t e = cudaSuccess;
  if (plan.splits > 1 || plan.reg) e = cudaMemsetAsync(base, 0, splitk_bytes, st);
  if (e != cudaSuccess) return record_cuda(e);
  e = launch_quantize_rows(act, scales, x, w->inverse, m, k, st);
  if (e != cudaSuccess) return record_cuda(e);

  CUtensorMap act_map;
  const CUtensorMap *wmap = nullptr;
  rc = make_map(&act_map, act, Kind::I8, k, m, static_cast<size_t>(k),
                plan.pair_sw ? plan.bn / 2 : plan.swap ? plan.bn : 128);
  if (rc) return rc;
  rc = weight_map(const_cast<htpg_weights *>(w), w_is_a ? 128 : box_rows_b(plan), &wmap);
  if (rc) return rc;
  GemmArgs a;
  a.M = m;
  a.N = n;
  a.K = k;
  a.out = out;
  a.ldo = ldo;
  a.mode = mode;
  a.channels = channels;
  a.row_scale = scales;
  a.col_scale = w->sw;
  a.col_corr = w->corr;
  a.col_sum7 = w->sum7;
  a.bias = bias;
  a.ws = wsk;
  a.ws_count = cnt;
  a.watchdog = d->watchdog;
  a.wk = w->wk;
  a.act = act;
  OutMaps out_maps;
  if (!w_is_a && mode != 3 && tma_store_ok(out, ldo)) {
    rc = make_out_map(&out_maps.map[0], out, m, n, ldo);
    if (rc) return rc;
    out_maps.count = 1;
    a.tma_store = 1;
  }
  e = w_is_a ? launch_gemm(plan, *wmap, act_map, out_maps, a, st)
             : launch_gemm(plan, act_map, *wmap, out_maps, a, st);
  return record_cuda(e);
}

void htpg::set_error_text(const char *text) { t_last_cuda_error = text ? text : ""; }

// ================================================================ one-call
namespace {

int cached_weights(Kind kind, const void *ptr, int k, int n, void *stream, htpg_weights **out, int qtype) {
  int dev = 0;
  cudaGetDevice(&dev);
  const CacheKey key(ptr, static_cast<int>(kind) + 100 * qtype, k, n, dev);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_cache.find(key);
    if (it != g_cache.end()) {
      *out = it->second;
      return HTPG_OK;
    }
  }
  htpg_weights *w = nullptr;
  const int rc = kind == Kind::QK0 ? htpg_qk0_weights_create(ptr, k, n, qtype, stream, &w)
                 : kind == Kind::I8
                     ? htpg_w8a8_weights_create(ptr, k, n, 0, 0, stream, &w)
                     : htpg_f16_weights_create(static_cast<const uint16_t *>(ptr), k, n, 0, 0, stream, &w);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  g_cache[key] = w;
  *out = w;
  return HTPG_OK;
}

}  // namespace

extern "C" void htpg_weight_cache_drop(const void *weights) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto it = g_cache.begin(); it != g_cache.end();) {
    if (std::get<0>(it->first) == weights) {
      htpg_weights_destroy(it->second);
      it = g_cache.erase(it);
    } else {
      ++it;
    }
  }
}

extern "C" void htpg_weight_cache_clear(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto &kv : g_cache) htpg_weights_destroy(kv.second);
  g_cache.clear();
}

extern "C" int htpg_w8a8_linear(float *out, const float *x, const void *constants, const float *bias,
                                int m, int k, int n, int channels, int mode, void *stream) {
  if (!out || !x || !constants || m < 1 || m > HTPG_W8A8_MAX_M || k < 32 || k > HTPG_W8A8_MAX_K ||
      n < 64 || n > HTPG_W8A8_MAX_N)
    return HTPG_EARGS;
  if (k % 32 || n % 64) return HTPG_EARGS;
  htpg_weights *w = nullptr;
  int rc = cached_weights(Kind::I8, constants, k, n, stream, &w);
  if (rc) return rc;
  return run_common(w, &out, 1, 0, x, bias, m, channels, mode, stream);
}

extern "C" int htpg_f16_linear(float *out, const float *x, const uint16_t *permuted_weight,
                               const float *bias, int m, int k, int n, int channels, int mode,
                               void *stream) {
  // argument checks in the reference's order and codes (mat_mul.c:939-951);
  // the diagnostic raw-accumulator mode is accepted here as well
  if (!out || !x || !permuted_weight || !m || !n || !k) return HTPG_EARGS;
  if (m < 1 || k < 1 || n < 1 || channels < 1 || channels > n || mode < 0 || mode > HTPG_MODE_RAW ||
      (mode != 3 && channels != n) || k % 32 || n % 32)
    return HTPG_ECAPACITY;
  if (m > HTPG_W8A8_MAX_M) return HTPG_ENOPLAN;
  htpg_weights *w = nullptr;
  int rc = cached_weights(Kind::F16, permuted_weight, k, n, stream, &w);
  if (rc) return rc;
  return run_common(w, &out, 1, 0, x, bias, m, channels, mode, stream);
}

// ================================================================ opcodes 2-4
namespace {

constexpr size_t kQCounterBytes = 64u * 1024u;  // stream-K arrival counters, kept zero

// Stream-private opcode 2-4 scratch: [counters | partial tiles | FP16 activations
// or the dequantised weight].  Zeroed when (re)allocated; the counters are
// left zero by every launch.
int qworkspace(Device *d, cudaStream_t st, size_t bytes, uint8_t **out) {
  Workspace &w = d->qws[st];
  if (w.bytes < bytes) {
    if (w.base) {
      cudaStreamSynchronize(st);
      cudaFree(w.base);
      w.base = nullptr;
      w.bytes = 0;
    }
    const size_t want = bytes + bytes / 4 + (1u << 20);
    if (cudaMalloc(&w.base, want) != cudaSuccess) {
      cudaGetLastError();
      return HTPG_ENOMEM;
    }
    if (cudaMemsetAsync(w.base, 0, want, st) != cudaSuccess) return HTPG_ELAUNCH;
    w.bytes = want;
  }
  *out = static_cast<uint8_t *>(w.base);
  return HTPG_OK;
}

bool qk0_type_ok(int qt) { return qk0_block_bytes(qt) != 0; }

}  // namespace

extern "C" size_t htpg_qk0_weight_bytes(int weight_type, int k, int n) {
  if (!qk0_type_ok(weight_type) || k < 32 || n < 32 || k % 32 || n % 32) return 0;
  return static_cast<size_t>(k) * static_cast<size_t>(n) / 256u * static_cast<size_t>(qk0_block_bytes(weight_type));
}

extern "C" int htpg_qk0_dequantize(uint16_t *w_nk, const void *weight, int k, int n, int weight_type,
                                   void *stream) {
  if (!w_nk || !weight || !qk0_type_ok(weight_type)) return HTPG_EARGS;
  if (k < 32 || n < 32 || k % 32 || n % 32) return HTPG_ECAPACITY;
  if ((reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(w_nk)) & 15u) return HTPG_ECONTROL;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  return record_cuda(launch_qk0_dequant(w_nk, static_cast<const uint8_t *>(weight), weight_type, k, n, 64, k,
                                        false, pick_stream(d, stream)));
}

extern "C" int htpg_qk0_weights_create(const void *weight, int k, int n, int weight_type, void *stream,
                                       htpg_weights **out) {
  if (!out) return HTPG_EARGS;
  *out = nullptr;
  if (!weight || !qk0_type_ok(weight_type)) return HTPG_EARGS;
  if (k < 32 || n < 32 || k % 32 || n % 32) return HTPG_ECAPACITY;
  if (reinterpret_cast<uintptr_t>(weight) & 15u) return HTPG_ECONTROL;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t st = pick_stream(d, stream);
  htpg_weights *w = new htpg_weights;
  w->kind = Kind::QK0;
  w->qtype = weight_type;
  w->k = k;
  w->ncols = n;
  w->n_total = n;
  w->device = d->ordinal;
  if (cudaMalloc(&w->wk, qk0_stage_records_bytes(weight_type, k, n)) != cudaSuccess) {
    cudaGetLastError();
    delete w;
    return HTPG_ENOMEM;
  }
  cudaError_t e = launch_qk0_repack(static_cast<uint8_t *>(w->wk), static_cast<const uint8_t *>(weight), weight_type,
                                    k, n, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) {
    htpg_weights_destroy(w);
    return record_cuda(e);
  }
  *out = w;
  return HTPG_OK;
}

extern "C" int htpg_qk0_run(const htpg_weights *w, float *out, const float *x, int m, void *stream) {
  if (!w || w->kind != Kind::QK0 || !out || !x) return HTPG_EARGS;
  const int k = w->k, n = w->ncols, qt = w->qtype;
  if (m < 1 || m > HTPG_W8A8_MAX_M) return HTPG_ECAPACITY;
  if ((reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(out) & 3u)) return HTPG_ECONTROL;
  Device *d;
  int rc = current_device(&d);
  if (rc) return rc;
  cudaStream_t st = pick_stream(d, stream);
  const uint8_t *records = static_cast<const uint8_t *>(w->wk);
  if (m > kQGemmMaxM) {
    // large M: the weight is dequantised once into K-major FP16 k-blocks and
    // the FP16 GEMM runs on it (its weight tiles load only after that pass)
    const size_t wbytes = kblock_bytes(Kind::F16, k, n);
    uint8_t *base = nullptr;
    {
      std::lock_guard<std::mutex> lk(g_mu);
      rc = qworkspace(d, st, kQCounterBytes + wbytes, &base);
      if (rc) return rc;
      const cudaError_t e = launch_qk0_dequant(reinterpret_cast<uint16_t *>(base + kQCounterBytes), records, qt, k, n,
                                               64LL * n, 64, true, st);
      if (e != cudaSuccess) return record_cuda(e);
    }
    htpg_weights f;
    f.kind = Kind::F16;
    f.k = k;
    f.ncols = n;
    f.n_total = n;
    f.device = d->ordinal;
    f.wk = base + kQCounterBytes;
    return run_common(&f, &out, 1, 0, x, nullptr, m, n, 0, stream, nullptr, nullptr, true);
  }
  std::lock_guard<std::mutex> lk(g_mu);
  const int qdec_mode = g_qdec.load();
  if (m <= 32 && (qdec_mode == 2 || (qdec_mode == 1 && qdec_serves(qt, m)))) {
    // decode shapes: the register-fed kernel (weights streamed into registers)
    const QDecPlan plan = plan_qdec(qt, m, n, k, d->sms);
    if (plan.grid == 0 || qdec_counter_bytes(plan) > kQCounterBytes || plan.smem > kQdMaxSlice) return HTPG_ENOPLAN;
    uint8_t *base = nullptr;
    rc = qworkspace(d, st, kQCounterBytes + align_up(qdec_partial_bytes(plan), 1024), &base);
    if (rc) return rc;
    QGemmArgs a;
    a.x = x;
    a.M = m;
    a.N = n;
    a.K = k;
    a.out = out;
    a.ldo = n;
    a.partials = reinterpret_cast<float *>(base + kQCounterBytes);
    a.counters = reinterpret_cast<uint32_t *>(base);
    a.watchdog = d->watchdog;
    return record_cuda(launch_qdec(qt, plan, records, a, st));
  }
  const QGemmPlan plan = plan_qgemm(qt, m, n, k, d->sms);
  if (qgemm_counter_bytes(plan) > kQCounterBytes) return HTPG_ENOPLAN;
  const size_t part = align_up(qgemm_partial_bytes(plan), 1024);
  uint8_t *base = nullptr;
  rc = qworkspace(d, st, kQCounterBytes + part, &base);
  if (rc) return rc;
  QGemmArgs a;
  a.x = x;
  a.M = m;
  a.N = n;
  a.K = k;
  a.out = out;
  a.ldo = n;
  a.partials = reinterpret_cast<float *>(base + kQCounterBytes);
  a.counters = reinterpret_cast<uint32_t *>(base);
  a.watchdog = d->watchdog;
  return record_cuda(launch_qgemm(qt, plan, records, a, st));
}

extern "C" int htpg_qk0_plan_info(int weight_type, int m, int n, int k, int sms, int64_t out[6]) {
  if (!out || !qk0_type_ok(weight_type) || m < 1 || m > kQGemmMaxM) return HTPG_EARGS;
  const QGemmPlan p = plan_qgemm(weight_type, m, n, k, sms);
  out[0] = p.bn;
  out[1] = p.tiles_a;
  out[2] = p.tiles_b;
  out[3] = p.kb_total;
  out[4] = p.grid;
  out[5] = static_cast<int64_t>(p.smem);
  return HTPG_OK;
}

extern "C" int htpg_qk0_decode_plan_info(int weight_type, int m, int n, int k, int sms, int64_t out[8]) {
  if (!out || !qk0_type_ok(weight_type) || m < 1 || m > 32 || n < 32 || k < 32 || n % 32 || k % 32 || sms < 1)
    return HTPG_EARGS;
  const QDecPlan p = plan_qdec(weight_type, m, n, k, sms);
  if (p.grid == 0) return HTPG_ENOPLAN;
  out[0] = p.per_sm;
  out[1] = p.nw;
  out[2] = p.ntiles;
  out[3] = p.ktiles;
  out[4] = p.splits;
  out[5] = p.grid;
  out[6] = static_cast<int64_t>(p.smem);
  out[7] = static_cast<int64_t>(qdec_smem_bytes(weight_type, p));
  return HTPG_OK;
}

extern "C" int htpg_qk0_linear(float *out, const float *x, const void *weight, int m, int k, int n,
                               int weight_type, void *stream) {
  if (!out || !x || !weight || !qk0_type_ok(weight_type)) return HTPG_EARGS;
  if (m < 1 || m > HTPG_W8A8_MAX_M || k < 32 || n < 32 || k % 32 || n % 32) return HTPG_ECAPACITY;
  htpg_weights *w = nullptr;
  int rc = cached_weights(Kind::QK0, weight, k, n, stream, &w, weight_type);
  if (rc) return rc;
  return htpg_qk0_run(w, out, x, m, stream);
}

// ================================================================ reference kernel names
// Synchronous like the reference kernels: return once the output is written.
namespace {

int finish_sync(int rc) {
  if (rc) return rc;
  return htpg_check_device(nullptr, nullptr);
}

}  // namespace

extern "C" int hmx_mat_mul_native_w8a8_profiled(float *dst, const float *activation,
                                                const uint8_t *constants, int m, int k, int n,
                                                struct NativeW8A8Profile *profile) {
  // reference admission (linear_w8a8.c:337-338) with the widened M/K limits
  if (!dst || !activation || !constants || m < 1 || m > HTPG_W8A8_MAX_M || k < 32 ||
      k > HTPG_W8A8_MAX_K || k % 32 || n < 64 || n > HTPG_W8A8_MAX_N || n % 64)
    return HTPG_EARGS;
  if (profile) {  // the caller's mode survives; every other field is rewritten
    const uint32_t mode = profile->mode;
    std::memset(profile, 0, sizeof(*profile));
    profile->mode = mode;
  }
  const auto t0 = std::chrono::steady_clock::now();
  htpg_weights *w = nullptr;
  int rc = cached_weights(Kind::I8, constants, k, n, nullptr, &w);
  if (rc) return rc;
  const auto t1 = std::chrono::steady_clock::now();
  const int prev = g_profiling;
  if (profile) g_profiling = 1;
  rc = finish_sync(run_common(w, &dst, 1, 0, activation, nullptr, m, 0, 0, nullptr));
  g_profiling = prev;
  if (profile && rc == HTPG_OK)
    htpg_w8a8_profile_fill(m, k, n, std::chrono::duration<double, std::milli>(t1 - t0).count(), profile);
  return rc;
}

// The trailer of a profiled opcode-15 request (reference op_reg.h:91-101,
// linear_w8a8.c:328-335, 396-399, 421-508), from the last run's phase events.
extern "C" int htpg_w8a8_profile_fill(int m, int k, int n, double setup_ms, struct NativeW8A8Profile *profile) {
  if (!profile) return HTPG_EARGS;
  const uint32_t mode = profile->mode;
  std::memset(profile, 0, sizeof(*profile));
  profile->mode = mode;
  const double tick_per_ms = 19200.0;  // the reference reports 19.2 MHz qtimer ticks
  profile->setup_ticks = static_cast<uint64_t>(setup_ms * tick_per_ms);
  profile->activation_ticks = static_cast<uint64_t>(t_phase_ms[0] * tick_per_ms);
  profile->hmx_ticks = static_cast<uint64_t>(t_phase_ms[1] * tick_per_ms);
  // weight loads and the output stores happen inside the GEMM launch: the
  // weight and output phases have no time of their own (0)
  if (mode == 2) profile->mac_ticks = profile->hmx_ticks;  // accumulation and readout are one launch
  if (mode == 3) {
    int dev = 0;
    cudaGetDevice(&dev);
    const GemmPlan p =
        plan_for(Kind::I8, m, n, k, dev >= 0 && dev < 16 && g_dev[dev].sms ? g_dev[dev].sms : 148, 0, 1);
    // low 16 bits: 64-row activation tiles per output tile; high 16 bits:
    // 64-column weight groups per output tile; bit 31 (table hit) stays 0,
    // every plan here comes from the shape-keyed planner
    const int act_rows = p.swap ? 64 : p.pair_sw ? p.bn : p.pair ? 256 : 128;
    const int w_cols = p.swap ? 128 : p.pair_sw ? 256 : p.bn;
    const uint32_t rows64 = static_cast<uint32_t>(act_rows / 64);
    const uint32_t cols64 = static_cast<uint32_t>(w_cols >= 64 ? w_cols / 64 : 1);
    profile->reserved = rows64 | (cols64 << 16);
    profile->mac_ticks = static_cast<uint64_t>(p.units);  // weight tiles (or tile pieces) loaded
    // weight bytes loaded: every k-block of every tile's weight columns once
    profile->readout_ticks = p.reg ? static_cast<uint64_t>(p.tiles_a) * 16u * p.kb_total * 128u
                                   : static_cast<uint64_t>(p.tiles_a) * p.tiles_b * p.splits *
                                         static_cast<uint64_t>(w_cols) * static_cast<uint64_t>(p.kb_per_split) * 128u;
  }
  return HTPG_OK;
}

extern "C" int hmx_mat_mul_native_w8a8(float *dst, const float *activation, const uint8_t *constants,
                                       int m, int k, int n) {
  return hmx_mat_mul_native_w8a8_profiled(dst, activation, constants, m, k, n, nullptr);
}

// The reference's CPU-epilogue form (linear_w8a8.c:205-227, 512-526): the
// unsigned-code INT32 accumulators leave as raw byte planes in the HMX export
// layout, the row scales and one batch descriptor go into the control block
// (htpg_w8a8_run_planes does both).
extern "C" int hmx_mat_mul_native_w8a8_cpu(float *dst, const float *activation,
                                           const uint8_t *constants, int m, int k, int n,
                                           struct W8A8CpuControl *control) {
  if (!control) return HTPG_ECONTROL;
  // argument checks as the reference kernel (linear_w8a8.c:337-338)
  if (!dst || !activation || !constants || m < 1 || m > 4096 || k < 32 || k > HTPG_W8A8_MAX_K || k % 32 ||
      n < 64 || n > HTPG_W8A8_MAX_N || n % 64)
    return HTPG_EARGS;
  htpg_weights *w = nullptr;
  int rc = cached_weights(Kind::I8, constants, k, n, nullptr, &w);
  if (rc) return rc;
  return htpg_w8a8_run_planes(w, dst, activation, m, control, nullptr);
}

extern "C" int hmx_mat_mul_f16_epilogue(float *dst, const float *activation, const uint16_t *weight,
                                        const float *bias, int m, int k, int n, int channels,
                                        int mode) {
  if (!dst || !activation || !weight || !m || !n || !k) return HTPG_EARGS;
  if (m < 1 || k < 1 || n < 1 || channels < 1 || channels > n || mode < 0 || mode > 3 ||
      (mode != 3 && channels != n) || k % 32 || n % 32)
    return HTPG_ECAPACITY;
  // the reference requires 128-byte aligned tensors (mat_mul.c:946-948)
  if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(activation) |
       reinterpret_cast<uintptr_t>(weight)) & 127u)
    return HTPG_ECONTROL;
  return finish_sync(htpg_f16_linear(dst, activation, weight, bias, m, k, n, channels, mode, nullptr));
}

// mat_mul.c:1601-1618: -1 for a missing operand, a zero size, K or N not a
// multiple of 32, an operand not 128-byte aligned or an unknown weight type.
extern "C" int hmx_mat_mul_permuted_qk_0_d16a32(float *dst, const float *activation,
                                                const uint8_t *permuted_weight, int m, int k, int n,
                                                int weight_type) {
  if (!dst || !activation || !permuted_weight || !m || !n || !k) return -1;
  if (k % 32 || n % 32) return -1;
  if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(activation) |
       reinterpret_cast<uintptr_t>(permuted_weight)) & 127u)
    return -1;
  if (!qk0_type_ok(weight_type) || m < 0 || k < 0 || n < 0) return -1;
  return finish_sync(htpg_qk0_linear(dst, activation, permuted_weight, m, k, n, weight_type, nullptr));
}

extern "C" int hmx_mat_mul_permuted_w16a32(float *dst, const float *activation,
                                           const uint16_t *permuted_weight, int m, int k, int n) {
  return hmx_mat_mul_f16_epilogue(dst, activation, permuted_weight, nullptr, m, k, n, n, 0);
}
