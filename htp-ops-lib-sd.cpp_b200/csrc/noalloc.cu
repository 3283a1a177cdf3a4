// htpg_w8a8_run_static: the W8A8 linear run for callers that cannot allocate
// device memory per call (a fixed memory budget, an external caching allocator
// that owns the device, or a loop that cannot absorb cudaMalloc's implicit
// device synchronisation).  Its scratch -- split-K area, activation codes, row
// scales -- is the file-scope static array below, one per device; nothing is
// allocated by any call.  The array lives in this translation unit alone; with
// CUDA's lazy module loading (the default, CUDA_MODULE_LOADING=LAZY) its module,
// and so the 32 MiB, is loaded on a device only once this entry point runs
// there, while eager loading places it on every device at start-up.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/htp_ops_b200.h"
#include "scratch_run.h"

namespace {

static_assert(HTPG_STATIC_SCRATCH_BYTES % 256 == 0, "scratch size keeps 256-byte alignment");
static_assert(HTPG_STATIC_SCRATCH_BYTES > htpg::kStaticSplitKBytes, "scratch holds the split-K area");

static __device__ __align__(256) unsigned char g_static_scratch[HTPG_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 16;
std::mutex g_setup_mu;
void *g_scratch_ptr[kMaxDevices] = {};

// One-time set-up per device, with that device current: the device address of
// this device's copy of the array.  Host code never uses the symbol itself as
// a device address.
int scratch_for_current_device(void **out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return HTPG_ELAUNCH;
  }
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    int rc = htpg_init(dev);  // device properties, architecture check, watchdog address
    if (rc != HTPG_OK) return rc;
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || !ptr) {
      htpg::set_error_text((std::string("cudaGetSymbolAddress(static scratch): ") +
                            cudaGetErrorString(e)).c_str());
      cudaGetLastError();
      return HTPG_ELAUNCH;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return HTPG_OK;
}

}  // namespace

extern "C" int htpg_w8a8_run_static(const htpg_weights *w, float *out, int ldo, const float *x,
                                    const float *bias, int m, int channels, int mode, void *stream) {
  void *scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != HTPG_OK) return rc;
  return htpg::w8a8_run_in_scratch(w, out, ldo, x, bias, m, channels, mode, stream, scratch,
                                   HTPG_STATIC_SCRATCH_BYTES);
}
