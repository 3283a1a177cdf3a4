// Host-side launchers of the device kernels (kernels.cu).  Internal to
// libhtp_ops_b200.so; the public surface is include/htp_ops_b200.h.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace htpg {

enum class Kind : int { I8 = 0, F16 = 1, QK0 = 2 };  // QK0: ggml-block stage records (never a GEMM kind)

// One GEMM launch: D[rows_a x rows_b] = A[rows_a x K] * B[rows_b x K]^T, both
// operands K-major in HBM and fetched by TMA.  Normal orientation: A = the
// activation (M rows), B = the weight (N rows).  Swapped (small M): A = the
// weight, B = the activation, so the 128-row MMA dimension runs over N.
struct GemmPlan {
  Kind kind = Kind::I8;
  bool swap = false;
  bool pair = false;     // CTA-pair tiles of 256 rows (tcgen05.mma.cta_group::2)
  bool pair_sw = false;  // pair tiles in the swapped orientation: A = the weight
                         // (256 columns per tile), B = the activation (bn rows)
  bool reg = false;      // register-fed decode kernel (decode.cu); swap is also set
  int chunks = 0;        // reg: contiguous (column group, k-block) ranges, one per CTA pass
  int bn = 256;          // MMA N (rows of B per tile)
  int splits = 1;        // K splits (I8 swapped only; exact INT32 reduction)
  int tiles_a = 0, tiles_b = 0;
  int kb_total = 0, kb_per_split = 0;
  int units = 0;         // tiles_a * tiles_b * splits, or full_units + tail tiles x tail_s
  int full_units = 0;    // swapped pair plans: units that are whole tiles (tail_s > 1)
  int tail_s = 1;        // swapped pair plans: pieces (K ranges) of each tile after full_units
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
  const void *wk = nullptr;          // the weight rows [KB][N][128 B] (register-fed decode)
  const void *act = nullptr;         // the activation codes [M][K] (register-fed decode)
  float one = 1.0f;                  // 1.0 as a runtime value (packed bias add, see finish2)
  int late_weights = 0;              // the weight is written by the kernels just before this
                                     // launch: no weight tile is loaded before the
                                     // programmatic-dependency wait (L2 prefetches only)
};

// Tensor map for TMA stores of a row-major FP32 output: `rows` x `cols`, row
// pitch ldo floats, 32 x 32 boxes with 128-byte swizzle.  Usable when `out` is
// 16-byte aligned and ldo is a multiple of 4.
inline bool tma_store_ok(const float *out, long long ldo) {
  return (reinterpret_cast<uintptr_t>(out) & 15u) == 0 && ldo % 4 == 0;
}

// Plan for an M x N x K problem (see plan_gemm in kernels.cu for the rules).
GemmPlan plan_gemm(Kind kind, int M, int N, int K, int num_sms);
// plan_gemm, with CTA-pair plans turned to the swapped orientation where the
// register-store epilogue serves the output (mode, number of destinations).
GemmPlan plan_for(Kind kind, int M, int N, int K, int num_sms, int mode, int n_outs, bool tail_split = true);
extern std::atomic<int> g_pair_direct;  // 0: CTA-pair plans keep the normal orientation
extern std::atomic<int> g_pair_tail;    // 0: swapped pair plans never cut their last round's tiles
// INT32 partial tiles of the pieces of a plan's split tail tiles (tail_s > 1).
size_t tail_slot_bytes(const GemmPlan &p);
// Bytes of split-K workspace (ws) and counters the plan needs.
size_t splitk_ws_bytes(const GemmPlan &p);
// Register-fed decode plan and launch (decode.cu).
void plan_decode_i8(GemmPlan &p, int M, int N, int K, int num_sms);
size_t decode_ws_bytes(const GemmPlan &p);
cudaError_t launch_decode_i8(const GemmPlan &p, const GemmArgs &a, cudaStream_t st);
extern std::atomic<int> g_decode_kernel;  // 0: register-fed decode for I8 M <= 16; 1: swapped tcgen05
// Read-only stream of `bytes` (a multiple of 32, 32-byte aligned) with the
// decode kernels' load policy (diagnostic: the HBM read ceiling).
cudaError_t launch_stream_read(const void *src, size_t bytes, int num_sms, cudaStream_t st);
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

// ---- opcodes 2-4: ggml-block weights dequantised to FP16 (qk0.cu) --------
// The weight is the reference's stream of K*N/256 super-blocks (8 FP16 scales +
// codes); super-block i dequantises to elements [256i, 256i+256) of the packed
// FP16 weight (element (k, n) at tile (n/32)*(K/32) + k/32, offset
// ((k%32)&~1)*32 + (n%32)*2 + (k&1)).  So one 32 x 32 tile is four
// consecutive super-blocks, super-block j of a tile holds k%32 in [8j, 8j+8)
// for all 32 columns, and its scale g covers the column half g%2 of the k pair
// g/2.
constexpr int kGgmlQ4_0 = 2, kGgmlQ8_0 = 8, kGgmlIQ4_NL = 20;
inline int qk0_block_bytes(int qt) {
  return qt == kGgmlQ8_0 ? 272 : (qt == kGgmlQ4_0 || qt == kGgmlIQ4_NL) ? 144 : 0;
}
// FP16 element (n, k) -> dst[(k/64)*stride_kb + n*stride_n + k%64].  src is
// the reference's stream, or (records) the stage records of
// launch_qk0_repack, whose zero padding also fills the k-block tail
// k in [K, 64*ceil(K/64)) (the K-major GEMM operand); from the stream that
// tail is left unwritten.
cudaError_t launch_qk0_dequant(uint16_t *dst, const uint8_t *src, int qt, int k, int n, long long stride_kb,
                               long long stride_n, bool records, cudaStream_t st);
// Stage records of the fused kernel (see qk0_repack_kernel): bytes, and the
// one-time reorder of the reference's stream into them.
size_t qk0_stage_records_bytes(int qt, int k, int n);
cudaError_t launch_qk0_repack(uint8_t *dst, const uint8_t *src, int qt, int k, int n, cudaStream_t st);
// Fused small-M GEMM: out[M][N] = f16(x) * dequant(W), the dequantised weight
// tile as the 128-row MMA operand, stream-K over (tile, k-block) iterations.
struct QGemmPlan {
  int bn = 16;                  // activation rows per tile (MMA N)
  int tiles_a = 0, tiles_b = 0; // 128-column weight tiles x activation-row tiles
  int kb_total = 0;             // 64-deep k-blocks
  long long iters = 0;          // tiles_a * tiles_b * kb_total
  int grid = 0;                 // CTAs (each owns a contiguous range of iterations)
  size_t smem = 0;
};
constexpr int kQGemmMaxM = 32;
QGemmPlan plan_qgemm(int qt, int M, int N, int K, int num_sms);
// Partial-tile slots (two per CTA) and per-tile arrival counters.
inline size_t qgemm_partial_bytes(const QGemmPlan &p) {
  return static_cast<size_t>(2) * p.grid * p.bn * 128 * 4;
}
inline size_t qgemm_counter_bytes(const QGemmPlan &p) {
  return static_cast<size_t>(p.tiles_a) * p.tiles_b * 4;
}
struct QGemmArgs {
  int M = 0, N = 0, K = 0;
  const float *x = nullptr;      // FP32 activations [M][K], 16-byte aligned
  float *out = nullptr;
  long long ldo = 0;
  float *partials = nullptr;     // qgemm_partial_bytes
  uint32_t *counters = nullptr;  // zero before the launch, left zero
  uint32_t *watchdog = nullptr;
};
// w: the stage records (launch_qk0_repack).
cudaError_t launch_qgemm(int qt, const QGemmPlan &p, const uint8_t *w, const QGemmArgs &a, cudaStream_t st);
// Register-fed decode for M <= 32 (qk0.cu, qdec_kernel): up to 16 32-column
// weight tiles x one k range per CTA, FP32 partials of the ranges summed in
// range order.  Partials: ntiles * splits * 32 * 8 nt floats; counters: ntiles.
constexpr size_t kQdMaxSlice = 64 * 1024;  // shared-memory bytes of the FP16 activation slice
struct QDecPlan {
  int nt = 1;          // 8-token MMA tiles (M <= 8: 1, M <= 16: 2, else 4)
  int ntiles = 0, ktiles = 0, splits = 1, grid = 0, pitch = 0;
  int nw = 16;         // weight tiles per CTA
  int per_sm = 1;      // CTAs resident per SM the plan is sized for
  size_t smem = 0;     // the activation slice
};
QDecPlan plan_qdec(int qt, int M, int N, int K, int num_sms);
size_t qdec_smem_bytes(int qt, const QDecPlan &p);  // the weight rings plus the activation slice
inline size_t qdec_partial_bytes(const QDecPlan &p) {
  return static_cast<size_t>(p.ntiles) * p.splits * 32 * 8 * p.nt * 4;
}
inline size_t qdec_counter_bytes(const QDecPlan &p) { return static_cast<size_t>(p.ntiles) * 4; }
cudaError_t launch_qdec(int qt, const QDecPlan &p, const uint8_t *w, const QGemmArgs &a, cudaStream_t st);
extern std::atomic<int> g_qdec;  // 1: the register-fed kernel where qdec_serves; 0: never; 2: every m <= 32
extern std::atomic<int> g_qdec_shape;  // 0: plan_qdec chooses; else CTAs per SM * 100 + tiles per CTA
// Where the register-fed kernel is the faster one: every type up to 32 tokens
// (LLM up / down projections, K x N = 4096 x 14336 and 14336 x 4096, back to
// back: 14.5-33 us against 34-43 us for the tcgen05 kernel).
inline bool qdec_serves(int qt, int m) {
  return (qt == kGgmlQ8_0 || qt == kGgmlQ4_0 || qt == kGgmlIQ4_NL) && m <= 32;
}

// Kernel launches issued since load (all launchers above count themselves).
uint64_t launches();
// Counts one launch when e is cudaSuccess; returns e.
cudaError_t counted(cudaError_t e);

}  // namespace htpg
