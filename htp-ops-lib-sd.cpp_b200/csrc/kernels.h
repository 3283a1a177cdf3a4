// Host-side launchers of the device kernels (kernels.cu).  Internal to
// libhtp_ops_b200.so; the public surface is include/htp_ops_b200.h.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace htpg {

enum class Kind : int { I8 = 0, F16 = 1 };

// One GEMM launch: D[rows_a x rows_b] = A[rows_a x K] * B[rows_b x K]^T, both
// operands K-major in HBM and fetched by TMA.  Normal orientation: A = the
// activation (M rows), B = the weight (N rows).  Swapped (small M): A = the
// weight, B = the activation, so the 128-row MMA dimension runs over N.
struct GemmPlan {
  Kind kind = Kind::I8;
  bool swap = false;
  bool pair = false;     // CTA-pair tiles of 256 rows (tcgen05.mma.cta_group::2)
  int bn = 256;          // MMA N (rows of B per tile)
  int splits = 1;        // K splits (I8 swapped only; exact INT32 reduction)
  int tiles_a = 0, tiles_b = 0;
  int kb_total = 0, kb_per_split = 0;
  int units = 0;         // tiles_a * tiles_b * splits
  int grid = 0;          // persistent CTAs
  size_t smem = 0;       // dynamic shared memory bytes
};

struct GemmArgs {
  int M = 0, N = 0, K = 0;        // logical problem (N = columns of this weight)
  float *out = nullptr;
  long long ldo = 0;              // elements between output rows
  int mode = 0, channels = 0;
  const float *row_scale = nullptr;  // I8: [M]
  const float *col_scale = nullptr;  // I8: [N]
  const int32_t *col_corr = nullptr; // I8: [N]
  const int32_t *col_sum7 = nullptr; // I8, plane export: [N] (sum_k w[n][k]) << 7
  const float *bias = nullptr;       // [N] or null
  int32_t *ws = nullptr;             // split-K accumulators
  uint32_t *ws_count = nullptr;      // split-K arrival counters (self-resetting)
  uint32_t *watchdog = nullptr;
  int tma_store = 0;                 // row-major output written by TMA through tmOut
};

// Tensor map for TMA stores of a row-major FP32 output: `rows` x `cols`, row
// pitch ldo floats, 32 x 32 boxes with 128-byte swizzle.  Usable when `out` is
// 16-byte aligned and ldo is a multiple of 4.
inline bool tma_store_ok(const float *out, long long ldo) {
  return (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && ldo % 4 == 0;
}

// Plan for an M x N x K problem (see plan_gemm in kernels.cu for the rules).
GemmPlan plan_gemm(Kind kind, int M, int N, int K, int num_sms);
// Bytes of split-K workspace (ws) and counters the plan needs.
size_t splitk_ws_bytes(const GemmPlan &p);
size_t splitk_count_bytes(const GemmPlan &p);
// Box rows of the A and B tensor maps for this plan.
// (swapped plans use the weight as A and the activation as B)
inline int box_rows_a(const GemmPlan &) { return 128; }
inline int box_rows_b(const GemmPlan &p) { return p.pair ? p.bn / 2 : p.bn; }

// Destinations of the row-major output: the epilogue stores every finished
// tile to each of them with TMA (the local output, and for the column-sharded
// multi-GPU run the same block of every peer's output).  count 0: no TMA
// stores (GemmArgs::tma_store is 0).
constexpr int kMaxOutputs = 8;
struct OutMaps {
  CUtensorMap map[kMaxOutputs];
  int count = 0;
};

cudaError_t launch_gemm(const GemmPlan &p, const CUtensorMap &tmA, const CUtensorMap &tmB,
                        const OutMaps &tmOut, const GemmArgs &a, cudaStream_t st);

cudaError_t launch_quantize_rows(int8_t *codes, float *scales, const float *x,
                                 const float *inverse, int m, int k, cudaStream_t st);
cudaError_t launch_to_f16(uint16_t *dst, const float *x, long long count, cudaStream_t st);
// Prepared weights are stored k-block-major: block kb (128 bytes of K: 128
// INT8 or 64 FP16 elements) of column n is row kb*ncols + n of a [KB*ncols][128 B]
// array, so the weight tile of one pipeline stage (consecutive columns, one
// k-block) is one contiguous run in HBM.  The last block is zero-padded.
inline int kblocks(Kind kind, int k) { return (k + (kind == Kind::I8 ? 127 : 63)) / (kind == Kind::I8 ? 128 : 64); }
inline size_t kblock_bytes(Kind kind, int k, int ncols) {
  return static_cast<size_t>(kblocks(kind, k)) * static_cast<size_t>(ncols) * 128u;
}
cudaError_t launch_repack_w8(int8_t *dst, const uint8_t *deep, int k, int n0, int ncols,
                             cudaStream_t st);
cudaError_t launch_colsum_corr(int32_t *corr, int32_t *sum7, const int8_t *wk, const int32_t *sums, int k,
                               int n0, int ncols, cudaStream_t st);
cudaError_t launch_check_ones(uint32_t *flag, const float *v, int count, cudaStream_t st);
cudaError_t launch_repack_f16(uint16_t *dst, const uint16_t *perm, int k, int n0, int ncols,
                              cudaStream_t st);

// Opcode-17 geometry (NativeConvParams without the buffers).
struct ConvGeom {
  int iw, ih, ic, ow, oh, kw, kh, sx, sy, px, py, dx, dy, kp, up;
};
// im2col rows [m0, m0 + rows) of one image (x: [ic][ih][iw] FP32) into
// a: [rows][kp] FP16 (round to nearest even), zero outside the (upsampled)
// image and for K columns past ic*kh*kw.
cudaError_t launch_im2col_f16(uint16_t *a, const float *x, const ConvGeom &g, int m0, int rows,
                              cudaStream_t st);

// Kernel launches issued since load (all launchers above count themselves).
uint64_t launches();

}  // namespace htpg
