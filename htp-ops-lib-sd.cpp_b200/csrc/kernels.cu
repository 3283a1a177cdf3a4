// Device kernels of the B200 linear-operator path.
//
//  * quantize_rows_*     per-row INT8 activation quantisation, bit-exact with
//                        the reference's IEEE restatement (linear_w8a8.c:34-128)
//  * to_f16_kernel       FP32 -> FP16 activation conversion (mat_mul.c:114-148)
//  * repack_*            one-time weight repacks from the reference layouts
//                        (HMX deep INT8, permuted FP16 tiles) to K-major rows
//  * gemm_kernel         warp-specialised persistent GEMM: TMA producer warp,
//                        single-thread tcgen05.mma issuer with double-buffered
//                        TMEM accumulators, four epilogue warps that apply the
//                        dequantisation / bias / activation / layout before
//                        the first HBM store.
#include <cuda_fp16.h>

#include <atomic>
#include <cstdio>


#include "kernels.h"
#include "ptx.cuh"
#include "quant.cuh"
#include "epilogue.cuh"

namespace htpg {

static std::atomic<uint64_t> g_launches{0};
uint64_t launches() { return g_launches.load(); }
cudaError_t counted(cudaError_t e) {
  if (e == cudaSuccess) g_launches.fetch_add(1);
  return e;
}

// ===================================================================== quant
// The per-element steps (scaled_input, quant_code, pack4, row_scale_of) are in
// quant.cuh.

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Rows are split over `TPR` threads (a warp or a whole block); each thread
// handles 8 consecutive elements per step (two float4 loads).
template <int TPR, int ROWS>
__global__ void __launch_bounds__(TPR *ROWS) quantize_rows_kernel(int8_t *__restrict__ codes,
                                                                 float *__restrict__ scales,
                                                                 const float *__restrict__ x,
                                                                 const float *__restrict__ inverse,
                                                                 int m, int k) {
  constexpr int kWarps = TPR / 32;
  __shared__ float red[ROWS][kWarps > 0 ? kWarps : 1];
  grid_dependents_launch();  // the GEMM may start its prologue and weight prefetch
  grid_dependency_wait();    // x may be the previous operator's output; the codes
                             // overwrite what the previous GEMM may still be reading
  const int local_row = threadIdx.x / TPR;
  const int t = threadIdx.x % TPR;
  const int row = blockIdx.x * ROWS + local_row;
  const bool valid = row < m;
  const float *xr = x + static_cast<size_t>(valid ? row : 0) * k;

  float amax = 0.0f;
  if (valid) {
    for (int c = t * 8; c < k; c += TPR * 8) {
      const float4 a = ld_dep_stream(reinterpret_cast<const float4 *>(xr + c));
      const float4 b = ld_dep_stream(reinterpret_cast<const float4 *>(xr + c + 4));
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(scaled_input(v[i], inverse, c + i)));
    }
  }
  amax = warp_max(amax);
  if (kWarps > 1) {
    if ((t & 31) == 0) red[local_row][t >> 5] = amax;
    __syncthreads();
    amax = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) amax = fmaxf(amax, red[local_row][w]);
  }
  if (!valid) return;
  const float scale = row_scale_of(amax);
  const float s = row_inverse_of(scale);
  if (t == 0) scales[row] = scale;
  int8_t *cr = codes + static_cast<size_t>(row) * k;
  for (int c = t * 8; c < k; c += TPR * 8) {
    const float4 a = ld_dep_stream(reinterpret_cast<const float4 *>(xr + c));
    const float4 b = ld_dep_stream(reinterpret_cast<const float4 *>(xr + c + 4));
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    int q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = quant_code(scaled_input(v[i], inverse, c + i), s);
    *reinterpret_cast<uint2 *>(cr + c) =
        make_uint2(pack4(q[0], q[1], q[2], q[3]), pack4(q[4], q[5], q[6], q[7]));
  }
}

// Rows of at most STEPS*256 elements: a warp per row that keeps the whole row
// in registers, so the row is read from HBM once and all of a lane's loads
// are in flight before the first use.
template <int STEPS>
__global__ void __launch_bounds__(256) quantize_rows_reg_kernel(int8_t *__restrict__ codes,
                                                                float *__restrict__ scales,
                                                                const float *__restrict__ x,
                                                                const float *__restrict__ inverse,
                                                                int m, int k) {
  grid_dependents_launch();  // the GEMM may start its prologue and weight prefetch
  grid_dependency_wait();    // x may be the previous operator's output; the codes
                             // overwrite what the previous GEMM may still be reading
  const int row = blockIdx.x * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= m) return;
  const float *xr = x + static_cast<size_t>(row) * k;
  float v[STEPS][8];
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int c = s * 256 + lane * 8;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (c < k) {
      a = ld_dep_stream(reinterpret_cast<const float4 *>(xr + c));
      b = ld_dep_stream(reinterpret_cast<const float4 *>(xr + c + 4));
    }
    v[s][0] = a.x; v[s][1] = a.y; v[s][2] = a.z; v[s][3] = a.w;
    v[s][4] = b.x; v[s][5] = b.y; v[s][6] = b.z; v[s][7] = b.w;
  }
  float amax = 0.0f;
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int c = s * 256 + lane * 8;
    if (c < k) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[s][i] = scaled_input(v[s][i], inverse, c + i);
        amax = fmaxf(amax, fabsf(v[s][i]));
      }
    }
  }
  amax = warp_max(amax);
  const float scale = row_scale_of(amax);
  const float inv_scale = row_inverse_of(scale);
  if (lane == 0) scales[row] = scale;
  int8_t *cr = codes + static_cast<size_t>(row) * k;
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const int c = s * 256 + lane * 8;
    if (c < k) {
      int q[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = quant_code(v[s][i], inv_scale);
      *reinterpret_cast<uint2 *>(cr + c) =
          make_uint2(pack4(q[0], q[1], q[2], q[3]), pack4(q[4], q[5], q[6], q[7]));
    }
  }
}

// Few long rows (decode): a 512-thread block per row that keeps the whole row
// in registers (J float4 per thread, J * 2048 >= k), so the row is read from
// HBM once, with all loads in flight together, and reduced across the block.
constexpr int kWideThreads = 512;
template <int J>
__global__ void __launch_bounds__(kWideThreads) quantize_rows_wide_kernel(int8_t *__restrict__ codes,
                                                                       float *__restrict__ scales,
                                                                       const float *__restrict__ x,
                                                                       const float *__restrict__ inverse,
                                                                       int m, int k) {
  __shared__ float red[kWideThreads / 32];
  grid_dependents_launch();  // the GEMM may start its prologue and weight prefetch
  grid_dependency_wait();    // x may be the previous operator's output; the codes
                             // overwrite what the previous GEMM may still be reading
  const int row = blockIdx.x;
  const int t = threadIdx.x;
  const float *xr = x + static_cast<size_t>(row) * k;
  float v[J][4];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = (j * kWideThreads + t) * 4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (c < k) a = ld_dep_stream(reinterpret_cast<const float4 *>(xr + c));
    v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
  }
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = (j * kWideThreads + t) * 4;
    if (c < k) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[j][i] = scaled_input(v[j][i], inverse, c + i);
        amax = fmaxf(amax, fabsf(v[j][i]));
      }
    }
  }
  amax = warp_max(amax);
  if ((t & 31) == 0) red[t >> 5] = amax;
  __syncthreads();
  amax = 0.0f;
#pragma unroll
  for (int w = 0; w < kWideThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float scale = row_scale_of(amax);
  const float inv_scale = row_inverse_of(scale);
  if (t == 0) scales[row] = scale;
  int8_t *cr = codes + static_cast<size_t>(row) * k;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int c = (j * kWideThreads + t) * 4;
    if (c < k)
      *reinterpret_cast<uint32_t *>(cr + c) =
          pack4(quant_code(v[j][0], inv_scale), quant_code(v[j][1], inv_scale), quant_code(v[j][2], inv_scale),
                quant_code(v[j][3], inv_scale));
  }
}

// Activation kernels are launched as programmatic dependents too: they may be
// scheduled while the previous operator's GEMM drains and wait (griddepcontrol)
// before reading its output.
template <typename Fn, typename... Args>
static cudaError_t launch_pdl(Fn fn, unsigned grid, unsigned block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(block, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, args...);
}

template <int STEPS>
static cudaError_t launch_reg(int8_t *codes, float *scales, const float *x, const float *inverse, int m,
                              int k, cudaStream_t st) {
  return launch_pdl(quantize_rows_reg_kernel<STEPS>, (m + 7) / 8, 256, st, codes, scales, x, inverse, m, k);
}

cudaError_t launch_quantize_rows(int8_t *codes, float *scales, const float *x,
                                 const float *inverse, int m, int k, cudaStream_t st) {
  // Many rows of at most 2048 elements: a register-resident warp per row.
  // Few rows, or rows longer than 2048 elements (up to 16384): a 512-thread
  // block per row that keeps the row in registers (one read from HBM).
  // Otherwise (fewer than 1184 rows of at most 2048): two passes per row,
  // the second from L1/L2.
  cudaError_t e;
  if (m <= 64 || (k > 2048 && k <= 8 * 2048)) {
    // decode shapes and long rows: one block per row, the row in registers
    const unsigned g = static_cast<unsigned>(m);
    switch ((k + 2047) / 2048) {
      case 1: e = launch_pdl(quantize_rows_wide_kernel<1>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
      case 2: e = launch_pdl(quantize_rows_wide_kernel<2>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
      case 3: e = launch_pdl(quantize_rows_wide_kernel<3>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
      case 4: e = launch_pdl(quantize_rows_wide_kernel<4>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
      case 5: e = launch_pdl(quantize_rows_wide_kernel<5>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
      case 6: e = launch_pdl(quantize_rows_wide_kernel<6>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
      case 7: e = launch_pdl(quantize_rows_wide_kernel<7>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
      default: e = launch_pdl(quantize_rows_wide_kernel<8>, g, kWideThreads, st, codes, scales, x, inverse, m, k); break;
    }
  } else if (k <= 2048 && m >= 1184) {
    switch ((k + 255) / 256) {
      case 1: e = launch_reg<1>(codes, scales, x, inverse, m, k, st); break;
      case 2: e = launch_reg<2>(codes, scales, x, inverse, m, k, st); break;
      case 3: e = launch_reg<3>(codes, scales, x, inverse, m, k, st); break;
      case 4: e = launch_reg<4>(codes, scales, x, inverse, m, k, st); break;
      case 5: e = launch_reg<5>(codes, scales, x, inverse, m, k, st); break;
      case 6: e = launch_reg<6>(codes, scales, x, inverse, m, k, st); break;
      case 7: e = launch_reg<7>(codes, scales, x, inverse, m, k, st); break;
      default: e = launch_reg<8>(codes, scales, x, inverse, m, k, st); break;
    }
  } else {
    e = launch_pdl(quantize_rows_kernel<256, 1>, static_cast<unsigned>(m), 256, st, codes, scales, x, inverse, m, k);
  }
  return counted(e != cudaSuccess ? e : cudaGetLastError());
}

__global__ void to_f16_kernel(uint16_t *__restrict__ dst, const float *__restrict__ x,
                              long long count) {
  grid_dependents_launch();
  grid_dependency_wait();
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= count) return;
  const float4 a = ld_dep_stream(reinterpret_cast<const float4 *>(x + i));
  const float4 b = ld_dep_stream(reinterpret_cast<const float4 *>(x + i + 4));
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = __half_as_ushort(__float2half_rn(v[2 * j]));
    const uint32_t hi = __half_as_ushort(__float2half_rn(v[2 * j + 1]));
    w[j] = lo | (hi << 16);
  }
  *reinterpret_cast<uint4 *>(dst + i) = make_uint4(w[0], w[1], w[2], w[3]);
}

cudaError_t launch_to_f16(uint16_t *dst, const float *x, long long count, cudaStream_t st) {
  const long long threads = (count + 7) / 8;
  const cudaError_t e = launch_pdl(to_f16_kernel, static_cast<unsigned>((threads + 255) / 256), 256, st, dst, x, count);
  return counted(e != cudaSuccess ? e : cudaGetLastError());
}

// ==================================================================== repack
// HMX deep N64 layout -> K-major rows dst[c][k] for columns n0+c.
__device__ __forceinline__ size_t deep_offset(int k_total, int n, int k) {
  return static_cast<size_t>(n / 64) * 64u * static_cast<size_t>(k_total) +
         static_cast<size_t>(k / 32) * 2048u + static_cast<size_t>((n % 64) / 32) * 1024u +
         static_cast<size_t>((k % 32) / 4) * 128u + static_cast<size_t>(n % 32) * 4u +
         static_cast<size_t>(k % 4);
}

__global__ void repack_w8_kernel(int8_t *__restrict__ dst, const uint8_t *__restrict__ deep, int k,
                                 int n0, int ncols) {
  const long long words = static_cast<long long>(ncols) * (k / 4);
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= words) return;
  const int c = static_cast<int>(i / (k / 4));
  const int kk = static_cast<int>(i % (k / 4)) * 4;
  const uint32_t v = __ldg(reinterpret_cast<const uint32_t *>(deep + deep_offset(k, n0 + c, kk)));
  const size_t row = static_cast<size_t>(kk / 128) * ncols + c;
  *reinterpret_cast<uint32_t *>(dst + row * 128u + kk % 128) = v;
}

cudaError_t launch_repack_w8(int8_t *dst, const uint8_t *deep, int k, int n0, int ncols,
                             cudaStream_t st) {
  const long long words = static_cast<long long>(ncols) * (k / 4);
  repack_w8_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, st>>>(dst, deep, k, n0,
                                                                               ncols);
  return counted(cudaGetLastError());
}

// corr[c] = (sum_k w[c][k] - sums[n0+c]) << 7 in wrapping INT32: the
// difference between the reference's zero-point correction, which uses the
// blob's stored column sums (linear_w8a8.c:159, 168), and the signed
// accumulation done here.  Zero for every blob whose sums are consistent.
__global__ void colsum_corr_kernel(int32_t *__restrict__ corr, int32_t *__restrict__ sum7,
                                   const int8_t *__restrict__ wk, const int32_t *__restrict__ sums, int k,
                                   int n0, int ncols) {
  const int c = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (c >= ncols) return;
  int s = 0;
  for (int i = lane * 4; i < k; i += 128) {
    // k-block-major: bytes [i, i+4) of column c sit in row (i/128)*ncols + c
    const uint32_t w = *reinterpret_cast<const uint32_t *>(
        wk + (static_cast<size_t>(i / 128) * ncols + c) * 128u + i % 128);
    s += static_cast<int8_t>(w & 0xff) + static_cast<int8_t>((w >> 8) & 0xff) +
         static_cast<int8_t>((w >> 16) & 0xff) + static_cast<int8_t>(w >> 24);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    const uint32_t diff = static_cast<uint32_t>(s) - static_cast<uint32_t>(sums[n0 + c]);
    corr[c] = static_cast<int32_t>(diff << 7);
    sum7[c] = static_cast<int32_t>(static_cast<uint32_t>(s) << 7);
  }
}

cudaError_t launch_colsum_corr(int32_t *corr, int32_t *sum7, const int8_t *wk, const int32_t *sums, int k,
                               int n0, int ncols, cudaStream_t st) {
  colsum_corr_kernel<<<(ncols + 7) / 8, 256, 0, st>>>(corr, sum7, wk, sums, k, n0, ncols);
  return counted(cudaGetLastError());
}

__global__ void check_ones_kernel(uint32_t *flag, const float *v, int count) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < count && __float_as_uint(v[i]) != 0x3f800000u) atomicOr(flag, 1u);
}

cudaError_t launch_check_ones(uint32_t *flag, const float *v, int count, cudaStream_t st) {
  check_ones_kernel<<<(count + 255) / 256, 256, 0, st>>>(flag, v, count);
  return counted(cudaGetLastError());
}

// Permuted FP16 tiles (element (k,n) at tile (n/32)*(K/32)+k/32, offset
// ((k%32)&~1)*32 + (n%32)*2 + (k&1)) -> K-major rows dst[c][k].  Elements k
// and k+1 (k even) are adjacent, so one 32-bit word moves a pair.
__global__ void repack_f16_kernel(uint16_t *__restrict__ dst, const uint16_t *__restrict__ perm,
                                  int k, int n0, int ncols) {
  const long long pairs = static_cast<long long>(ncols) * (k / 2);
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= pairs) return;
  const int c = static_cast<int>(i / (k / 2));
  const int kk = static_cast<int>(i % (k / 2)) * 2;
  const int n = n0 + c;
  const size_t tile = static_cast<size_t>(n / 32) * static_cast<size_t>(k / 32) + kk / 32;
  const size_t off = tile * 1024u + static_cast<size_t>(kk % 32) * 32u + static_cast<size_t>(n % 32) * 2u;
  const uint32_t v = __ldg(reinterpret_cast<const uint32_t *>(perm + off));
  const size_t row = static_cast<size_t>(kk / 64) * ncols + c;
  *reinterpret_cast<uint32_t *>(dst + row * 64u + kk % 64) = v;
}

cudaError_t launch_repack_f16(uint16_t *dst, const uint16_t *perm, int k, int n0, int ncols,
                              cudaStream_t st) {
  const long long pairs = static_cast<long long>(ncols) * (k / 2);
  repack_f16_kernel<<<static_cast<unsigned>((pairs + 255) / 256), 256, 0, st>>>(dst, perm, k, n0,
                                                                                ncols);
  return counted(cudaGetLastError());
}

// ====================================================================== conv
// im2col of opcode 17 (the reference gathers the same values, mat_mul.c:2230-2290):
// row t (output position oy*ow + ox), column col = ci*kh*kw + ky*kw + kx reads
// the nearest-upsampled input at (ox*sx - px + kx*dx, oy*sy - py + ky*dy).
// A block transposes a tile of 128 rows x 32 columns through shared memory:
// consecutive threads gather consecutive rows of one column (consecutive x,
// coalesced), then the FP16 tile leaves as 64-byte row segments.
constexpr int kI2cRows = 128, kI2cCols = 32, kI2cPitch = kI2cCols + 2;  // halves per staged row
__global__ void __launch_bounds__(256) im2col_f16_kernel(uint16_t *__restrict__ a, const float *__restrict__ x,
                                                        ConvGeom g, int m0, int rows) {
  __shared__ uint16_t tile[kI2cRows * kI2cPitch];
  __shared__ int col_ci[kI2cCols], col_ky[kI2cCols], col_kx[kI2cCols];
  grid_dependents_launch();  // the GEMM may start its prologue and weight prefetch
  const int r0 = blockIdx.x * kI2cRows, c0 = blockIdx.y * kI2cCols;
  if (threadIdx.x < kI2cCols) {
    const int col = c0 + threadIdx.x, khw = g.kw * g.kh;
    const int ci = col / khw, rem = col - ci * khw, ky = rem / g.kw;
    col_ci[threadIdx.x] = ci;
    col_ky[threadIdx.x] = ky * g.dy;
    col_kx[threadIdx.x] = (rem - ky * g.kw) * g.dx;
  }
  __syncthreads();
  const int tr = threadIdx.x % kI2cRows, tc = threadIdx.x / kI2cRows;  // row, column phase (0..1)
  const int r = r0 + tr;
  const bool row_ok = r < rows;
  const int t = m0 + (row_ok ? r : 0);
  const int oy = t / g.ow, ox = t - oy * g.ow;
  const int xbase = ox * g.sx - g.px, ybase = oy * g.sy - g.py;
  const int wu = g.iw * g.up, hu = g.ih * g.up;
  const int ush = g.up == 2 ? 1 : 0;  // nearest upsample: source index = index >> 1
#pragma unroll 4
  for (int cc = tc; cc < kI2cCols; cc += 2) {
    const int ci = col_ci[cc], xx = xbase + col_kx[cc], yy = ybase + col_ky[cc];
    const float v = (row_ok && ci < g.ic && xx >= 0 && xx < wu && yy >= 0 && yy < hu)
                        ? ld_dep(x + (static_cast<size_t>(ci) * g.ih + (yy >> ush)) * g.iw + (xx >> ush))
                        : 0.0f;
    tile[tr * kI2cPitch + cc] = __half_as_ushort(__float2half_rn(v));
  }
  __syncthreads();
  // 128 rows x 64 bytes = 512 segments of 16 bytes, two per thread
#pragma unroll
  for (int q = threadIdx.x; q < kI2cRows * 4; q += 256) {
    const int rr = q >> 2, part = q & 3;
    if (r0 + rr >= rows) continue;
    const uint32_t *src = reinterpret_cast<const uint32_t *>(tile + rr * kI2cPitch + part * 8);
    *reinterpret_cast<uint4 *>(a + static_cast<size_t>(r0 + rr) * g.kp + c0 + part * 8) =
        make_uint4(src[0], src[1], src[2], src[3]);
  }
}

cudaError_t launch_im2col_f16(uint16_t *a, const float *x, const ConvGeom &g, int m0, int rows,
                              cudaStream_t st) {
  const dim3 grid(static_cast<unsigned>((rows + kI2cRows - 1) / kI2cRows), static_cast<unsigned>(g.kp / kI2cCols));
  im2col_f16_kernel<<<grid, 256, 0, st>>>(a, x, g, m0, rows);
  return counted(cudaGetLastError());
}

// ====================================================================== GEMM
// Sixteen epilogue warps: four per TMEM lane quadrant, so each SM sub-partition
// interleaves four independent chunk pipelines (the epilogue is latency-bound).
constexpr int kEpiWarps = 16;
constexpr int kEpiPerQuadrant = kEpiWarps / 4;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 64 + kEpiThreads;         // warp 0 TMA, warp 1 MMA/TMEM, 2..17 epilogue
constexpr int kRowBytes = 128;                     // one K block = one 128-byte swizzle row
constexpr int kPrefetchBytes = 512 * 1024;         // L2 warm-up per CTA while the activation pass runs
// Per epilogue warp: a 32 x 32 FP32 output tile staged with 128-byte swizzle
// (row r at r*128 bytes, 16-byte chunk j at position j ^ (r & 7)), the source
// layout of the TMA store and conflict-free for row- and column-wise access;
// plus 96 floats of per-column parameters for each of its (up to two) chunks.
constexpr int kWarpScratch = 32 * 32;              // floats per epilogue warp (4 KiB)
constexpr int kWarpParams = 192;                   // floats per epilogue warp (two chunks)
constexpr int kEpiSmem = kEpiWarps * (kWarpScratch + kWarpParams) * 4;

constexpr int kSmemLimit = 232448;  // opt-in dynamic shared memory per block on sm_100
constexpr int kMaxStages = 12;      // the 256-byte barrier block holds 2 x 12 + 5 barriers
// Epilogue shared memory: swapped (small-M) tiles need only the parameter
// slots, the normal orientation also the staging tiles of the TMA stores.
__host__ __device__ constexpr int epi_smem_for(bool swap) {
  return swap ? kEpiWarps * kWarpParams * 4 : kEpiSmem;
}
// k-blocks per pipeline stage.  Swapped (small-M) tiles move 16 KB of weights
// per k-block behind only four N = 16/32 MMAs; a stage's MMA group and its
// release commit cost about 0.4 us however small, so a stage of one k-block
// caps the weight stream near 3.4 TB/s and two k-blocks per stage raise that
// to about 4.9 TB/s (stream + MMA + commit loop measured in isolation).
__host__ __device__ constexpr int kbs_for(bool swap) { return swap ? 2 : 1; }
// As many pipeline stages as fit beside the epilogue's shared memory.
__host__ __device__ constexpr int stages_for(int bn, bool swap = false) {
  return (kSmemLimit - 1024 - 256 - epi_smem_for(swap)) / (kbs_for(swap) * (128 + bn) * kRowBytes) < kMaxStages
             ? (kSmemLimit - 1024 - 256 - epi_smem_for(swap)) / (kbs_for(swap) * (128 + bn) * kRowBytes)
             : kMaxStages;
}
__host__ __device__ constexpr int tmem_cols_for(int bn) {
  return 2 * bn <= 32 ? 32 : 2 * bn <= 64 ? 64 : 2 * bn <= 128 ? 128 : 2 * bn <= 256 ? 256 : 512;
}
__host__ __device__ constexpr size_t smem_bytes_for(int bn, bool swap = false) {
  return 1024 /* alignment slack */ + static_cast<size_t>(stages_for(bn, swap)) * kbs_for(swap) * (128 + bn) * kRowBytes +
         static_cast<size_t>(epi_smem_for(swap)) + 256 /* barriers, tmem slot, flags */;
}
static_assert((2 * kMaxStages + 5) * 8 + 12 <= 256, "barrier block");
static_assert(smem_bytes_for(256) <= kSmemLimit && smem_bytes_for(128) <= kSmemLimit &&
                  smem_bytes_for(64) <= kSmemLimit && smem_bytes_for(32) <= kSmemLimit &&
                  smem_bytes_for(16, true) <= kSmemLimit && smem_bytes_for(32, true) <= kSmemLimit,
              "shared memory budget");

struct SmemLayout {
  uint8_t *a;          // STAGES x KBS x 128 rows x 128 B
  uint8_t *b;          // STAGES x KBS x BN rows x 128 B
  float *scratch;      // per epilogue warp: the 32 x 32 staging tile (1024-byte aligned)
  float *params;       // per epilogue warp: 96 floats of column parameters
  uint64_t *full, *empty, *tfull, *tempty, *mma_done;
  uint32_t *tmem_slot;
  uint32_t *flag;            // split-K "this CTA finishes the tile"
  volatile uint32_t *abort;  // sticky: some wait of this CTA gave up
};

template <int BN, int STAGES, bool SWAP = false>
__device__ __forceinline__ SmemLayout carve(uint8_t *raw) {
  SmemLayout L;
  uint8_t *p = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  L.a = p;
  p += STAGES * kbs_for(SWAP) * 128 * kRowBytes;
  L.b = p;
  p += STAGES * kbs_for(SWAP) * BN * kRowBytes;
  L.scratch = reinterpret_cast<float *>(p);  // swapped tiles stage nothing
  if (!SWAP) p += kEpiWarps * kWarpScratch * 4;
  L.params = reinterpret_cast<float *>(p);
  p += kEpiWarps * kWarpParams * 4;
  uint64_t *bars = reinterpret_cast<uint64_t *>(p);
  L.full = bars;
  L.empty = bars + STAGES;
  L.tfull = bars + 2 * STAGES;
  L.tempty = bars + 2 * STAGES + 2;
  L.mma_done = bars + 2 * STAGES + 4;
  L.tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
  L.flag = L.tmem_slot + 1;
  L.abort = L.tmem_slot + 2;
  return L;
}

struct Unit {
  int ta, tb, ks;
};
__device__ __forceinline__ Unit decode_unit(int u, int tiles_b, int splits) {
  Unit w;
  w.ta = u / (tiles_b * splits);
  const int r = u % (tiles_b * splits);
  w.tb = r / splits;
  w.ks = r % splits;
  return w;
}

struct KernelParams {
  GemmArgs a;
  int tiles_a, tiles_b, splits, kb_total, kb_per_split, units;
  int full_units = 0, tail_s = 1;  // CTA-pair plans: whole-tile units, then pieces of the tail tiles
};

// A CTA-pair unit: the tile and its k-block range.  Units below full_units are
// whole tiles; the rest cut each remaining (tail) tile into tail_s pieces of
// consecutive k-blocks, piece `part` of tile t at unit full_units + (t -
// full_units) * tail_s + part.  Units go round-robin to the pairs, and
// full_units is a multiple of the pair count, so every piece is its pair's
// last unit and all pieces of the tail run side by side.
struct PairUnit {
  int tile, kb0, kb1, part;
};
__device__ __forceinline__ PairUnit pair_unit(const KernelParams &P, int u) {
  PairUnit r;
  if (u < P.full_units) {
    r.tile = u;
    r.kb0 = 0;
    r.kb1 = P.kb_total;
    r.part = 0;
    return r;
  }
  const int j = u - P.full_units;
  const int t = j / P.tail_s;
  r.tile = P.full_units + t;
  r.part = j - t * P.tail_s;
  r.kb0 = P.kb_total * r.part / P.tail_s;
  r.kb1 = P.kb_total * (r.part + 1) / P.tail_s;
  return r;
}

// Tail-piece hand-off counters: a piece publishes the INT32 sums of the
// chunks other pieces own and then arrives on their counters (release, made
// cumulative by the epilogue barrier before it); it waits for the other
// pieces' arrivals on its own counter (acquire) before reading their sums.
__device__ __forceinline__ void arrive_release(uint32_t *count) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(count) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire(const uint32_t *count) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(count) : "memory");
  return v;
}
// Bounded wait for *count to reach `target` (the time limit and the CTA's
// abort flag as in mbar_wait).
__device__ __forceinline__ bool wait_count(const uint32_t *count, uint32_t target, uint32_t *watchdog,
                                           volatile uint32_t *abort) {
  if (load_acquire(count) >= target) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    __nanosleep(32);
    if (load_acquire(count) >= target) return true;
    if ((spin & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        atomicOr(watchdog, kWatchSplitK);
        *abort = 1u;
        return false;
      }
    }
  }
}

// Everything an epilogue warp needs for one unit.
struct EpiCtx {
  const GemmArgs *g;
  const KernelParams *P;
  const OutMaps *tmOut;
  SmemLayout L;
  float *scr;        // this warp's staging tile
  float *prm;        // this warp's column-parameter slots
  uint32_t t_row;    // TMEM address of lane quadrant q, accumulator buffer
  uint32_t full_bar, full_parity;  // accumulator-full barrier of this unit
  uint32_t empty_bar;              // accumulator-free barrier (the leader's, for pairs)
  bool empty_remote;               // empty_bar is in the leader CTA of the pair
  Unit w;
  int row0;                        // first output row held by this CTA's TMEM lanes
  int q, part, lane, epi_t;        // part: which of the quadrant's four warps
};


// Normal orientation: TMEM lane = activation row m, column = weight column n.
// The four warps of a lane quadrant take every fourth 32-column chunk.  The row
// scale and the per-column parameters are loaded before the accumulator wait,
// so their latency hides behind the MMAs.  A warp reads all of its chunks from
// TMEM at once and hands the accumulator buffer back to the MMA warp before it
// does any arithmetic or stores, so the next-but-one tile's MMAs never wait for
// this tile's epilogue.  Returns whether the wait succeeded (the buffer has
// then been released).
template <Kind KIND, int BN, int MODE, bool BIAS>
__device__ __forceinline__ bool epilogue_normal(const EpiCtx &c) {
  constexpr int kChunks = BN / 32;
  // BN < 128: one chunk for the first kChunks warps of a quadrant; BN >= 128:
  // exactly kMine chunks for every warp
  constexpr int kMine = (kChunks + kEpiPerQuadrant - 1) / kEpiPerQuadrant;
  static_assert(kMine * 96 <= kWarpParams, "parameter slots per warp");
  const GemmArgs &g = *c.g;
  const bool active = c.part < kChunks;
  if (!active) {
    const bool ok = mbar_wait(c.full_bar, c.full_parity, g.watchdog, kWatchEpilogue, c.L.abort);
    tc_fence_after();
    if (ok && c.lane == 0) {
      if (c.empty_remote)
        mbar_arrive_cluster_relaxed(c.empty_bar);
      else
        mbar_arrive(c.empty_bar);
    }
    return ok;
  }
  const int m = c.row0 + c.q * 32 + c.lane;
  const bool m_ok = m < g.M;
  const float rs = (KIND == Kind::I8 && m_ok) ? ld_dep(g.row_scale + m) : 0.0f;
  float psw[kMine], pb[kMine];
  int pcr[kMine];
#pragma unroll
  for (int i = 0; i < kMine; ++i) {
    const int nl = c.w.tb * BN + (c.part + kEpiPerQuadrant * i) * 32 + c.lane;
    const bool ok = nl < g.N;
    psw[i] = (KIND == Kind::I8 && ok) ? __ldg(g.col_scale + nl) : 0.0f;
    pcr[i] = (KIND == Kind::I8 && ok) ? __ldg((MODE == 5 ? g.col_sum7 : g.col_corr) + nl) : 0;
    pb[i] = (BIAS && ok) ? ld_dep(g.bias + nl) : 0.0f;
  }
  const bool ok = mbar_wait(c.full_bar, c.full_parity, g.watchdog, kWatchEpilogue, c.L.abort);
  tc_fence_after();
  if (!ok) return false;
  // per-column parameters -> prm[96 i + 0..95] (scale, correction, bias), read
  // back as broadcasts; the previous unit's reads are complete (syncwarp)
  float *prm = c.prm;
  __syncwarp();
#pragma unroll
  for (int i = 0; i < kMine; ++i) {
    if (KIND == Kind::I8) {
      prm[96 * i + c.lane] = psw[i];
      prm[96 * i + 32 + c.lane] = __int_as_float(pcr[i]);
    }
    if (BIAS) prm[96 * i + 64 + c.lane] = pb[i];
  }
  uint32_t r[kMine][32];
#pragma unroll
  for (int i = 0; i < kMine; ++i) tmem_ld32(c.t_row + (c.part + kEpiPerQuadrant * i) * 32, r[i]);
  tmem_ld_wait();
  tc_fence_before();
  __syncwarp();
  if (c.lane == 0) {
    if (c.empty_remote)
      mbar_arrive_cluster_relaxed(c.empty_bar);
    else
      mbar_arrive(c.empty_bar);
  }
  float *scr = c.scr;
  const bool tma = MODE != 3 && g.tma_store;
  const int mbase = c.row0 + c.q * 32;
#pragma unroll
  for (int i = 0; i < kMine; ++i) {
    const int n0 = c.w.tb * BN + (c.part + kEpiPerQuadrant * i) * 32;
    const int nl = n0 + c.lane;
    const bool nl_ok = nl < g.N;
    const float *pi = prm + 96 * i;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f), c4 = s4, b4 = s4;
      if (KIND == Kind::I8) {
        s4 = *reinterpret_cast<const float4 *>(pi + j);
        c4 = *reinterpret_cast<const float4 *>(pi + 32 + j);
      }
      if (BIAS) b4 = *reinterpret_cast<const float4 *>(pi + 64 + j);
      r[i][j + 0] = __float_as_uint(finish<KIND, MODE, BIAS>(r[i][j + 0], __float_as_int(c4.x), s4.x, rs, b4.x));
      r[i][j + 1] = __float_as_uint(finish<KIND, MODE, BIAS>(r[i][j + 1], __float_as_int(c4.y), s4.y, rs, b4.y));
      r[i][j + 2] = __float_as_uint(finish<KIND, MODE, BIAS>(r[i][j + 2], __float_as_int(c4.z), s4.z, rs, b4.z));
      r[i][j + 3] = __float_as_uint(finish<KIND, MODE, BIAS>(r[i][j + 3], __float_as_int(c4.w), s4.w, rs, b4.w));
    }
    if (MODE == 3) {
      // channel-major out[n*ldo + m]: lanes hold consecutive m -> coalesced
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + j;
        if (m_ok && n < g.channels) g.out[static_cast<long long>(n) * g.ldo + m] = __uint_as_float(r[i][j]);
      }
    } else if (MODE == 5) {
      // byte planes: 32 contiguous bytes per plane for this row's 32 columns
      if (m_ok && n0 < g.N) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          uint32_t wv[8];
#pragma unroll
          for (int q = 0; q < 8; ++q)
            wv[q] = ((r[i][4 * q] >> (8 * p)) & 0xffu) | (((r[i][4 * q + 1] >> (8 * p)) & 0xffu) << 8) |
                    (((r[i][4 * q + 2] >> (8 * p)) & 0xffu) << 16) | (((r[i][4 * q + 3] >> (8 * p)) & 0xffu) << 24);
          uint8_t *d = plane_dst(g.out, g.ldo, g.M, m, n0, p);
          if (g.tma_store) {  // 16-byte aligned rows
            reinterpret_cast<uint4 *>(d)[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            reinterpret_cast<uint4 *>(d)[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) d[q] = static_cast<uint8_t>(wv[q >> 2] >> (8 * (q & 3)));
          }
        }
      }
    } else {
      // row-major: stage the 32 x 32 tile (128-byte swizzle), then one TMA
      // store, or (unaligned output) coalesced 128-byte row stores.  The
      // previous chunk's TMA store must be done reading the staging tile.
      if (tma && c.lane == 0) bulk_wait_read_all();
      __syncwarp();
      char *row = reinterpret_cast<char *>(scr) + c.lane * 128;
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4)
        *reinterpret_cast<uint4 *>(row + ((j4 ^ (c.lane & 7)) << 4)) =
            make_uint4(r[i][4 * j4], r[i][4 * j4 + 1], r[i][4 * j4 + 2], r[i][4 * j4 + 3]);
      if (tma) {
        fence_proxy_async_smem();
        __syncwarp();
        if (c.lane == 0) {
          for (int d = 0; d < c.tmOut->count; ++d) tma_store_2d(&c.tmOut->map[d], smem_u32(scr), n0, mbase);
          bulk_commit();
        }
      } else {
        __syncwarp();
        const char *base = reinterpret_cast<const char *>(scr);
        const int cpos = c.lane >> 2, cofs = (c.lane & 3) * 4;
#pragma unroll 8
        for (int rr = 0; rr < 32; ++rr) {
          const int mr = mbase + rr;
          const float val =
              *reinterpret_cast<const float *>(base + rr * 128 + ((cpos ^ (rr & 7)) << 4) + cofs);
          if (mr < g.M && nl_ok) g.out[static_cast<long long>(mr) * g.ldo + nl] = val;
        }
        __syncwarp();
      }
    }
  }
  return true;
}

// Swapped orientation (small M): TMEM lane = weight column n, column = activation
// row m (BN <= 32).  One warp per lane quadrant holds the data; all epilogue
// warps take part in the split-K barriers.  Returns whether the wait succeeded.
template <Kind KIND, int BN, int MODE, bool BIAS>
__device__ __forceinline__ bool epilogue_swap(const EpiCtx &c) {
  const GemmArgs &g = *c.g;
  const KernelParams &P = *c.P;
  const bool owner = c.part == 0;
  const int n = c.w.ta * 128 + c.q * 32 + c.lane;
  const bool n_ok = n < g.N;
  const bool c_ok = mbar_wait(c.full_bar, c.full_parity, g.watchdog, kWatchEpilogue, c.L.abort);
  tc_fence_after();
  uint32_t r[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) r[j] = 0u;
  if (c_ok && owner) {
    if (BN == 16) {
      uint32_t r16[16];
      tmem_ld16(c.t_row, r16);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 16; ++j) r[j] = r16[j];
    } else {
      tmem_ld32(c.t_row, r);
      tmem_ld_wait();
    }
  }
  bool fin = c_ok;
  if (P.splits > 1) {
    // exact INT32 split-K: partials meet in HBM; the last CTA of the tile
    // finishes it and leaves the accumulators and counter zeroed
    const int tile = c.w.ta * P.tiles_b + c.w.tb;
    int32_t *ws = g.ws + (static_cast<size_t>(tile) * 128 + c.q * 32 + c.lane) * BN;
    if (c_ok && owner) {
#pragma unroll
      for (int j = 0; j < BN; ++j) atomicAdd(ws + j, static_cast<int32_t>(r[j]));
      __threadfence();
    }
    named_bar_sync(1, kEpiThreads);
    if (c.epi_t == 0) {
      uint32_t last = 0u;
      if (!*c.L.abort) {
        const uint32_t prev = atomicAdd(g.ws_count + tile, 1u);
        last = (prev == static_cast<uint32_t>(P.splits - 1)) ? 1u : 0u;
      }
      *c.L.flag = last;
    }
    named_bar_sync(1, kEpiThreads);
    fin = c_ok && *c.L.flag != 0u;
    if (fin && owner) {
      __threadfence();
#pragma unroll
      for (int j = 0; j < BN; ++j) {
        r[j] = static_cast<uint32_t>(__ldcg(ws + j));
        ws[j] = 0;
      }
      if (c.epi_t == 0) g.ws_count[tile] = 0u;
    }
    named_bar_sync(1, kEpiThreads);
  }
  if (!fin || !owner) return c_ok;
  float *scr = c.prm;  // the row scales of this tile's (at most 32) activation rows
  const int mrow = c.w.tb * BN + c.lane;
  scr[c.lane] = (KIND == Kind::I8 && mrow < g.M) ? ld_dep(g.row_scale + mrow) : 0.0f;
  __syncwarp();
  if (!n_ok) return c_ok;
  float sw = 0.0f, bn_ = 0.0f;
  int32_t cr = 0;
  if (KIND == Kind::I8) {
    sw = __ldg(g.col_scale + n);
    cr = __ldg((MODE == 5 ? g.col_sum7 : g.col_corr) + n);
  }
  if (BIAS) bn_ = ld_dep(g.bias + n);
#pragma unroll
  for (int j = 0; j < BN; ++j) {
    const int m = c.w.tb * BN + j;
    if (m >= g.M) break;
    const float v = finish<KIND, MODE, BIAS>(r[j], cr, sw, scr[j], bn_);
    if (MODE == 5) {
      const uint32_t u = __float_as_uint(v);
#pragma unroll
      for (int p = 0; p < 4; ++p) *plane_dst(g.out, g.ldo, g.M, m, n, p) = static_cast<uint8_t>(u >> (8 * p));
    } else if (MODE == 3) {
      if (n < g.channels) g.out[static_cast<long long>(n) * g.ldo + m] = v;
    } else {
      g.out[static_cast<long long>(m) * g.ldo + n] = v;
    }
  }
  return c_ok;
}

template <Kind KIND, int BN, bool SWAP, int MODE, bool BIAS>
__device__ __forceinline__ bool epilogue_unit(const EpiCtx &c) {
  if constexpr (SWAP)
    return epilogue_swap<KIND, BN, MODE, BIAS>(c);
  else
    return epilogue_normal<KIND, BN, MODE, BIAS>(c);
}

template <Kind KIND, int BN, bool SWAP>
__device__ __forceinline__ bool epilogue_dispatch(const EpiCtx &c, int mode, bool bias) {
  switch (mode * 2 + (bias ? 1 : 0)) {
    case 0: return epilogue_unit<KIND, BN, SWAP, 0, false>(c);
    case 1: return epilogue_unit<KIND, BN, SWAP, 0, true>(c);
    case 2: return epilogue_unit<KIND, BN, SWAP, 1, false>(c);
    case 3: return epilogue_unit<KIND, BN, SWAP, 1, true>(c);
    case 4: return epilogue_unit<KIND, BN, SWAP, 2, false>(c);
    case 5: return epilogue_unit<KIND, BN, SWAP, 2, true>(c);
    case 6: return epilogue_unit<KIND, BN, SWAP, 3, false>(c);
    case 7: return epilogue_unit<KIND, BN, SWAP, 3, true>(c);
    case 10: return epilogue_unit<KIND, BN, SWAP, 5, false>(c);
    default: return epilogue_unit<KIND, BN, SWAP, 4, false>(c);
  }
}

template <Kind KIND, int BN, bool SWAP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ OutMaps tmOut, const KernelParams P) {
  constexpr int STAGES = stages_for(BN, SWAP);
  constexpr int TCOLS = tmem_cols_for(BN);
  constexpr int KBS = kbs_for(SWAP);                       // k-blocks per stage
  constexpr uint32_t kKbBytes = (128 + BN) * kRowBytes;    // both operands of one k-block
  constexpr int kElemsPerRow = KIND == Kind::I8 ? 128 : 64;
  constexpr uint32_t kIdesc = KIND == Kind::I8 ? idesc_i8(128, BN) : idesc_f16(128, BN);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
  static_assert(!SWAP || BN <= 32, "swapped tiles hold at most 32 activation rows");

  extern __shared__ uint8_t smem_raw[];
  const SmemLayout L = carve<BN, STAGES, SWAP>(smem_raw);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const GemmArgs &g = P.a;
  uint32_t *wd = g.watchdog;
  // the next operator's kernels may be scheduled now (they wait for this one
  // before they read anything it writes)
  grid_dependents_launch();
  if (threadIdx.x == 32) {  // the descriptor fetch overlaps the set-up below
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&L.full[s]), 1);
      mbar_init(smem_u32(&L.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&L.tfull[b]), 1);
      mbar_init(smem_u32(&L.tempty[b]), kEpiWarps);
    }
    mbar_init(smem_u32(L.mma_done), 1);
    *L.abort = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(L.tmem_slot), TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *L.tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      // The weights do not depend on the activation pass that may still be
      // running: put this CTA's first weight tiles into the ring (and warm the
      // L2 with the next ones) before waiting for it.
      // A stage holds KBS k-blocks (sub-tile j of stage s at s*KBS + j); the
      // last stage of a unit may hold fewer.
      int pre = 0;  // leading stages of the first unit whose weight tiles are in flight
      if (blockIdx.x < P.units) {
        const Unit w = decode_unit(blockIdx.x, P.tiles_b, P.splits);
        const int kb0 = w.ks * P.kb_per_split;
        const int kb1 = min(kb0 + P.kb_per_split, P.kb_total);
        pre = g.late_weights ? 0 : min(STAGES, (kb1 - kb0 + KBS - 1) / KBS);
        for (int i = 0; i < pre; ++i) {
          const uint32_t fb = smem_u32(&L.full[i]);
          const int kbi = kb0 + i * KBS, nk = min(KBS, kb1 - kbi);
          mbar_arrive_expect_tx(fb, nk * kKbBytes);
          for (int j = 0; j < nk; ++j) {
            if (SWAP)
              tma_load_2d(smem_u32(L.a + (i * KBS + j) * 128 * kRowBytes), &tmA, fb, 0, (kbi + j) * g.N + w.ta * 128);
            else
              tma_load_2d(smem_u32(L.b + (i * KBS + j) * BN * kRowBytes), &tmB, fb, 0, (kbi + j) * g.N + w.tb * BN);
          }
        }
        const int kb2 = min(kb1, kb0 + kPrefetchBytes / ((SWAP ? 128 : BN) * kRowBytes));
        for (int kb = kb0 + pre * KBS; kb < kb2; ++kb) {
          if (SWAP)
            tma_prefetch_l2_2d(&tmA, 0, kb * g.N + w.ta * 128);
          else
            tma_prefetch_l2_2d(&tmB, 0, kb * g.N + w.tb * BN);
        }
      }
      grid_dependency_wait();
      int s = 0;
      uint32_t ph = 0;
      int last_phase[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) last_phase[i] = i < pre ? 0 : -1;
      bool ok = true;
      bool first = true;
      for (int u = blockIdx.x; ok && u < P.units; u += gridDim.x, first = false) {
        const Unit w = decode_unit(u, P.tiles_b, P.splits);
        const int kb0 = w.ks * P.kb_per_split;
        const int kb1 = min(kb0 + P.kb_per_split, P.kb_total);
        for (int kbs = kb0; kbs < kb1; kbs += KBS) {
          if (!mbar_wait(smem_u32(&L.empty[s]), ph ^ 1u, wd, kWatchProducer, L.abort)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&L.full[s]);
          const int nk = min(KBS, kb1 - kbs);
          // the weight operand (A when swapped, else B) is k-block-major:
          // its box starts at row kb * N + first column
          const bool weight_done = first && (kbs - kb0) / KBS < pre;
          if (!weight_done) mbar_arrive_expect_tx(fb, nk * kKbBytes);
          for (int j = 0; j < nk; ++j) {
            const int kb = kbs + j, sub = s * KBS + j;
            if (SWAP) {
              if (!weight_done)
                tma_load_2d(smem_u32(L.a + sub * 128 * kRowBytes), &tmA, fb, 0, kb * g.N + w.ta * 128);
              tma_load_2d(smem_u32(L.b + sub * BN * kRowBytes), &tmB, fb, kb * kElemsPerRow, w.tb * BN);
            } else {
              tma_load_2d(smem_u32(L.a + sub * 128 * kRowBytes), &tmA, fb, kb * kElemsPerRow, w.ta * 128);
              if (!weight_done)
                tma_load_2d(smem_u32(L.b + sub * BN * kRowBytes), &tmB, fb, 0, kb * g.N + w.tb * BN);
            }
          }
          last_phase[s] = static_cast<int>(ph);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Never leave the CTA with a TMA copy still landing in its shared memory.
      for (int i = 0; i < STAGES; ++i)
        if (last_phase[i] >= 0)
          mbar_wait(smem_u32(&L.full[i]), static_cast<uint32_t>(last_phase[i]), wd, kWatchProducer,
                    L.abort);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      grid_dependency_wait();  // bounded waits start once the operands can exist
      int s = 0;
      uint32_t ph = 0;
      uint32_t iter = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < P.units; u += gridDim.x, ++iter) {
        const Unit w = decode_unit(u, P.tiles_b, P.splits);
        const int kb0 = w.ks * P.kb_per_split;
        const int kb1 = min(kb0 + P.kb_per_split, P.kb_total);
        const uint32_t buf = iter & 1u;
        const uint32_t acc_ph = (iter >> 1) & 1u;
        if (!mbar_wait(smem_u32(&L.tempty[buf]), acc_ph ^ 1u, wd, kWatchMma, L.abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kbs = kb0; kbs < kb1; kbs += KBS) {
          if (!mbar_wait(smem_u32(&L.full[s]), ph, wd, kWatchMma, L.abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nk = min(KBS, kb1 - kbs);
          for (int j = 0; j < nk; ++j) {
            const uint32_t a_addr = smem_u32(L.a + (s * KBS + j) * 128 * kRowBytes);
            const uint32_t b_addr = smem_u32(L.b + (s * KBS + j) * BN * kRowBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t da = umma_desc_sw128(a_addr + kk * 32);
              const uint64_t db = umma_desc_sw128(b_addr + kk * 32);
              const uint32_t accumulate = (kbs > kb0 || j > 0 || kk > 0) ? 1u : 0u;
              if (KIND == Kind::I8)
                umma_i8(d_tmem, da, db, kIdesc, accumulate);
              else
                umma_f16(d_tmem, da, db, kIdesc, accumulate);
            }
          }
          tc_commit(smem_u32(&L.empty[s]));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit(smem_u32(&L.tfull[buf]));
      }
      // All MMAs of this thread complete before TMEM can be released.
      tc_commit(smem_u32(L.mma_done));
      mbar_wait(smem_u32(L.mma_done), 0, wd, kWatchMma, L.abort);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    EpiCtx c;
    c.g = &g;
    c.P = &P;
    c.tmOut = &tmOut;
    c.L = L;
    c.q = warp & 3;                            // TMEM lane quadrant of this warp
    c.part = (warp - 2) / 4;                   // which of the quadrant's four warps
    c.lane = lane;
    c.epi_t = threadIdx.x - 64;
    c.scr = L.scratch + (warp - 2) * kWarpScratch;
    c.prm = L.params + (warp - 2) * kWarpParams;
    const bool has_bias = g.bias != nullptr;
    grid_dependency_wait();  // row scales come from the activation pass
    uint32_t iter = 0;
    // No early exit: all epilogue warps run the same iterations so their
    // named barriers always match; after a failed wait the unit's work is
    // skipped (the watchdog word reports the failure).
    for (int u = blockIdx.x; u < P.units; u += gridDim.x, ++iter) {
      c.w = decode_unit(u, P.tiles_b, P.splits);
      const uint32_t buf = iter & 1u;
      const uint32_t acc_ph = (iter >> 1) & 1u;
      c.full_bar = smem_u32(&L.tfull[buf]);
      c.full_parity = acc_ph;
      c.row0 = c.w.ta * 128;
      c.t_row = tmem_base + (static_cast<uint32_t>(c.q * 32) << 16) + buf * BN;
      c.empty_bar = smem_u32(&L.tempty[buf]);
      c.empty_remote = false;
      const bool ok = epilogue_dispatch<KIND, BN, SWAP>(c, g.mode, has_bias);
      if constexpr (SWAP) {
        // this warp's TMEM reads of the buffer are complete (tcgen05.wait::ld);
        // the normal orientation releases the buffer inside its epilogue
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(c.empty_bar);
      }
    }
    if (lane == 0) bulk_wait_all();  // output stores of this warp have landed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TCOLS);
  }
}

// ================================================================ 2-SM GEMM
// A CTA pair (cluster of two) computes one 256 x BN tile with
// tcgen05.mma.cta_group::2.  CTA r loads A rows [ta*256 + r*128, +128) and B
// rows [tb*BN + r*BN/2, +BN/2) into its own shared memory (no multicast); the
// leader (rank 0) issues the MMAs, which read both CTAs' halves; CTA r's TMEM
// receives output rows ta*256 + r*128 .. +127 (all BN columns) and its own
// epilogue warps finish them.  Per SM this moves 16 KB instead of 24 KB of
// operands through shared memory per 128 x 256 x 32 MMA step, which is what
// lets the tensor pipe run past the shared-memory bandwidth ceiling of the
// single-CTA tile.
// Epilogue shared memory of the pair kernel: the staging tiles and column
// parameters of the TMA-store epilogue, or (swapped orientation, stores from
// registers) only the per-warp row-scale slots.
__host__ __device__ constexpr int epi2_smem_for(bool sw) { return sw ? kEpiWarps * kWarpParams * 4 : kEpiSmem; }
__host__ __device__ constexpr int stages2_for(int bn, bool sw = false) {
  return (kSmemLimit - 1024 - 256 - epi2_smem_for(sw)) / ((128 + bn / 2) * kRowBytes) < 10
             ? (kSmemLimit - 1024 - 256 - epi2_smem_for(sw)) / ((128 + bn / 2) * kRowBytes)
             : 10;
}
__host__ __device__ constexpr size_t smem2_bytes_for(int bn, bool sw = false) {
  return 1024 + static_cast<size_t>(stages2_for(bn, sw)) * (128 + bn / 2) * kRowBytes +
         static_cast<size_t>(epi2_smem_for(sw)) + 256;
}
static_assert(smem2_bytes_for(256) <= kSmemLimit && smem2_bytes_for(128) <= kSmemLimit &&
                  smem2_bytes_for(256, true) <= kSmemLimit && smem2_bytes_for(128, true) <= kSmemLimit,
              "shared memory budget (pair)");

// Shared-memory carve-up of the pair kernel (one k-block per stage).
template <int BH, int STAGES, bool SW>
__device__ __forceinline__ SmemLayout carve2(uint8_t *raw) {
  SmemLayout L;
  uint8_t *p = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  L.a = p;
  p += STAGES * 128 * kRowBytes;
  L.b = p;
  p += STAGES * BH * kRowBytes;
  L.scratch = reinterpret_cast<float *>(p);  // the swapped orientation stages nothing
  if (!SW) p += kEpiWarps * kWarpScratch * 4;
  L.params = reinterpret_cast<float *>(p);
  p += kEpiWarps * kWarpParams * 4;
  uint64_t *bars = reinterpret_cast<uint64_t *>(p);
  L.full = bars;
  L.empty = bars + STAGES;
  L.tfull = bars + 2 * STAGES;
  L.tempty = bars + 2 * STAGES + 2;
  L.mma_done = bars + 2 * STAGES + 4;
  L.tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 5);
  L.flag = L.tmem_slot + 1;
  L.abort = L.tmem_slot + 2;
  return L;
}

// Swapped orientation of the pair tile (weights are the 256-row MMA operand,
// activations the MMA N): TMEM lane = output column n, TMEM column = activation
// row m.  Each epilogue warp owns 32 columns (its lane quadrant) and BN/4 rows
// (its part) of every unit.  Per row, the warp's 32 lanes store 32
// consecutive FP32 outputs: one 128-byte line per store instruction, straight
// from registers, so the output never passes through shared memory.  Column
// scale, correction and bias are per-thread constants, the rows' scales are
// read as shared-memory broadcasts, and both are fetched one unit ahead so
// their global-load latency hides behind the current unit's arithmetic.  The
// whole unit loop lives here (one dispatch on the epilogue mode per launch).
// Output stores marked as streaming (evict-first in the L2): the output is
// written once and not read by this kernel, and with the default policy its
// stream (403 MB for C4) evicts the activation-code tiles that later tiles
// read again.  Measured on C4: operator 158.2 -> 154.1 us (interleaved
// medians); no change where the output fits in the L2.
__device__ __forceinline__ void st_stream(float *p, float v) {
  asm volatile("st.global.cs.f32 [%0], %1;" ::"l"(p), "f"(v));
}
template <Kind KIND, int BN, int MODE, bool BIAS>
__device__ __forceinline__ void epilogue_loop_sw(const GemmArgs &g, const KernelParams &P, const SmemLayout &L,
                                                 float *rs, uint32_t tmem_base, int q, int part, int lane,
                                                 int pair, int npairs, uint32_t rank, uint32_t peer_abort) {
  constexpr int kTok = BN / kEpiPerQuadrant;  // rows (TMEM columns) per warp and unit: 64 or 32
  constexpr int kCh = kTok / 32;
  static_assert(kTok <= kWarpParams, "row-scale slot per warp");
  const uint32_t ldo4 = static_cast<uint32_t>(g.ldo) * 4u;  // bytes per output row (< 2^31 by the shape limits)
  const uint64_t one2 = pk2(g.one, g.one);
  float f_sw = 0.0f, f_bv = 0.0f, f_rs[kCh];
  int32_t f_cr = 0;
  auto fetch = [&](int u) {
    const Unit w = decode_unit(pair_unit(P, u).tile, P.tiles_b, 1);
    const int n = w.ta * 256 + static_cast<int>(rank) * 128 + q * 32 + lane;
    const int m0 = w.tb * BN + part * kTok;
    const bool ok = n < g.N;
    f_sw = (KIND == Kind::I8 && ok) ? __ldg(g.col_scale + n) : 0.0f;
    f_cr = (KIND == Kind::I8 && ok) ? __ldg(g.col_corr + n) : 0;
    f_bv = (BIAS && ok) ? ld_dep(g.bias + n) : 0.0f;
#pragma unroll
    for (int i = 0; i < kCh; ++i) {
      const int m = m0 + 32 * i + lane;
      f_rs[i] = (KIND == Kind::I8 && m < g.M) ? ld_dep(g.row_scale + m) : 0.0f;
    }
  };
  if (pair < P.units) fetch(pair);
  const int epi_t = static_cast<int>(threadIdx.x) - 64;  // among the CTA's epilogue threads
  uint32_t iter = 0;
  for (int u = pair; u < P.units; u += npairs, ++iter) {
    const PairUnit pu = pair_unit(P, u);
    const Unit w = decode_unit(pu.tile, P.tiles_b, 1);
    const uint32_t buf = iter & 1u;
    const int n = w.ta * 256 + static_cast<int>(rank) * 128 + q * 32 + lane;
    const bool n_ok = n < g.N;
    const int m0 = w.tb * BN + part * kTok;
    // Tail pieces (reduce-scatter of their INT32 sums): piece k owns the
    // tile's 32-row chunks c with c % tail_s == k, so each warp owns at most
    // one of its two chunks.  Every piece stores the chunks it does not own in
    // its slot [BN rows][128 columns] per (tail tile, piece, CTA), arrives on
    // the owners' counters (per tail tile, owner piece and CTA), waits for the
    // other pieces' arrivals on its own counter, adds their slots' rows of
    // its chunks to its accumulator and finishes those rows.
    const bool piece = u >= P.full_units;
    const int tt = pu.tile - P.full_units;
    auto count = [&](int owner) { return g.ws_count + (tt * P.tail_s + owner) * 2 + static_cast<int>(rank); };
    auto slot = [&](int k) {
      return g.ws + (static_cast<size_t>((tt * P.tail_s + k) * 2 + static_cast<int>(rank)) * BN + part * kTok) * 128 +
             q * 32 + lane;
    };
    auto owner_of = [&](int i) { return (part * kCh + i) % P.tail_s; };  // chunk i of this warp
    // this unit's parameters (the f_ registers are refilled for the next unit below)
    const float sw = f_sw, bv = f_bv;
    const uint64_t bias2 = pk2(bv, bv);
    const int32_t cr = f_cr;
    __syncwarp();  // the previous unit's reads of the row-scale slot are complete
#pragma unroll
    for (int i = 0; i < kCh; ++i) rs[32 * i + lane] = f_rs[i];
    __syncwarp();
    if (u + npairs < P.units) fetch(u + npairs);
    const bool ok = mbar_wait(smem_u32(&L.tfull[buf]), (iter >> 1) & 1u, g.watchdog, kWatchEpilogue, L.abort);
    tc_fence_after();
    if (!ok) {
      st_shared_cluster(peer_abort, 1u);
      if (!piece) return;  // a piece's warps all meet at its barrier below, failed or not
    }
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN + part * kTok;
    if (piece) {
      if (ok) {
        int32_t *sl = slot(pu.part);
#pragma unroll 1
        for (int i = 0; i < kCh; ++i) {
          if (owner_of(i) == pu.part) continue;
          uint32_t r[32];
          tmem_ld32(t_row + 32 * i, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) __stcg(sl + (32 * i + j) * 128, static_cast<int32_t>(r[j]));
        }
      }
      named_bar_sync(1, kEpiThreads);  // every slot store of this CTA precedes the arrivals
      if (epi_t == 0) {
        bool got = *L.abort == 0u;
        if (got)
          for (int o = 0; o < P.tail_s; ++o)
            if (o != pu.part) arrive_release(count(o));
        got = got && wait_count(count(pu.part), static_cast<uint32_t>(P.tail_s - 1), g.watchdog, L.abort);
        if (got) *count(pu.part) = 0u;  // left zero for the next launch (every arrival is in)
        *L.flag = got ? 1u : 0u;
      }
      named_bar_sync(1, kEpiThreads);
      if (!ok || *L.flag == 0u) {
        st_shared_cluster(peer_abort, 1u);
        return;
      }
    }
    // One 32-row chunk at a time (the code of one chunk stays small next to
    // the MMA issuer's loop in the instruction caches); the accumulator goes
    // back to the pair leader's MMA issuer once the last chunk is in registers.
#pragma unroll 1
    for (int i = 0; i < kCh; ++i) {
      const bool mine = !piece || owner_of(i) == pu.part;
      uint32_t r[32];
      if (mine) {
        tmem_ld32(t_row + 32 * i, r);
        tmem_ld_wait();
      }
      if (i == kCh - 1) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(mapa_shared(smem_u32(&L.tempty[buf]), 0));
      }
      if (!mine) continue;
      if (piece) {
        for (int k = 0; k < P.tail_s; ++k) {
          if (k == pu.part) continue;
          const int32_t *sl = slot(k) + 32 * i * 128;
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = static_cast<uint32_t>(static_cast<int32_t>(r[j]) + __ldcg(sl + j * 128));
        }
      }
      const int mb = m0 + 32 * i;
      if (!n_ok || mb >= g.M) continue;
      char *base = reinterpret_cast<char *>(g.out + static_cast<long long>(mb) * g.ldo + n);
      const float *rsi = rs + 32 * i;
      auto row = [&](int j) {
        return reinterpret_cast<float *>(base + static_cast<unsigned long long>(ldo4) * static_cast<unsigned>(j));
      };
      if (mb + 32 <= g.M) {
        if constexpr (KIND == Kind::I8) {
          const uint64_t sw2 = pk2(sw, sw);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 s4 = *reinterpret_cast<const float4 *>(rsi + 4 * j4);
            float o0, o1, o2, o3;
            finish2<MODE, BIAS>(r[4 * j4], r[4 * j4 + 1], cr, sw2, s4.x, s4.y, bias2, one2, o0, o1);
            finish2<MODE, BIAS>(r[4 * j4 + 2], r[4 * j4 + 3], cr, sw2, s4.z, s4.w, bias2, one2, o2, o3);
            st_stream(row(4 * j4), o0);
            st_stream(row(4 * j4 + 1), o1);
            st_stream(row(4 * j4 + 2), o2);
            st_stream(row(4 * j4 + 3), o3);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) *row(j) = finish<KIND, MODE, BIAS>(r[j], 0, 0.0f, 0.0f, bv);
        }
      } else {
        const int valid = g.M - mb;
#pragma unroll
        for (int j = 0; j < 32; ++j)  // constant indices keep r[] in registers
          if (j < valid) *row(j) = finish<KIND, MODE, BIAS>(r[j], cr, sw, KIND == Kind::I8 ? rsi[j] : 0.0f, bv);
      }
    }
  }
}

template <Kind KIND, int BN>
__device__ __forceinline__ void epilogue_loop_sw_dispatch(const GemmArgs &g, const KernelParams &P,
                                                          const SmemLayout &L, float *rs, uint32_t tmem_base, int q,
                                                          int part, int lane, int pair, int npairs, uint32_t rank,
                                                          uint32_t peer_abort) {
#define HTPG_SW_LOOP(M_, B_) \
  epilogue_loop_sw<KIND, BN, M_, B_>(g, P, L, rs, tmem_base, q, part, lane, pair, npairs, rank, peer_abort)
  switch (g.mode * 2 + (g.bias ? 1 : 0)) {
    case 0: HTPG_SW_LOOP(0, false); break;
    case 1: HTPG_SW_LOOP(0, true); break;
    case 2: HTPG_SW_LOOP(1, false); break;
    case 3: HTPG_SW_LOOP(1, true); break;
    case 4: HTPG_SW_LOOP(2, false); break;
    case 5: HTPG_SW_LOOP(2, true); break;
    default: HTPG_SW_LOOP(4, false); break;
  }
#undef HTPG_SW_LOOP
}

// SW (swapped orientation): A = the weight (tile ta: columns ta*256 + r*128
// in CTA r), B = the activation codes (tile tb: rows tb*BN + r*BN/2), and the
// epilogue stores from registers (epilogue_pair_sw).  Otherwise A = the
// activation codes (rows ta*256 + r*128), B = the weight (columns tb*BN +
// r*BN/2) and the epilogue leaves through TMA stores.
template <Kind KIND, int BN, bool SW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ OutMaps tmOut, const KernelParams P) {
  constexpr int BH = BN / 2;  // B rows held by each CTA
  constexpr int STAGES = stages2_for(BN, SW);
  constexpr int TCOLS = tmem_cols_for(BN);
  constexpr uint32_t kStageBytes = (128 + BH) * kRowBytes;  // per CTA
  constexpr int kElemsPerRow = KIND == Kind::I8 ? 128 : 64;
  constexpr uint32_t kIdesc = KIND == Kind::I8 ? idesc_i8(256, BN) : idesc_f16(256, BN);
  static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");

  extern __shared__ uint8_t smem_raw[];
  const SmemLayout L = carve2<BH, STAGES, SW>(smem_raw);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const GemmArgs &g = P.a;
  uint32_t *wd = g.watchdog;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<uint32_t *>(L.abort)), rank ^ 1u);
  grid_dependents_launch();  // the next operator's kernels may be scheduled now
  if (threadIdx.x == 32) {     // the descriptor fetch overlaps the set-up below
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  // a failed wait also tells the peer CTA, whose waits then return at once
  auto wait = [&](uint32_t bar, uint32_t parity, uint32_t bit) {
    const bool ok = mbar_wait(bar, parity, wd, bit, L.abort);
    if (!ok) st_shared_cluster(peer_abort, 1u);
    return ok;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&L.full[s]), 1);
      mbar_init(smem_u32(&L.empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&L.tfull[b]), 1);
      mbar_init(smem_u32(&L.tempty[b]), 2 * kEpiWarps);  // epilogue warps of both CTAs
    }
    mbar_init(smem_u32(L.mma_done), 1);
    *L.abort = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(L.tmem_slot), TCOLS);
    tmem_relinquish_pair();
  }
  // both CTAs' barriers exist before either CTA signals the other
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *L.tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      // this CTA's part of the weight tile of k-block kb and unit w (into ring
      // stage s), and its part of the activation tile
      auto load_weight = [&](int s, int kb, const Unit &w, uint32_t fb) {
        if (SW)
          tma_load_2d_pair(smem_u32(L.a + s * 128 * kRowBytes), &tmA, fb, 0,
                           kb * g.N + w.ta * 256 + static_cast<int>(rank) * 128);
        else
          tma_load_2d_pair(smem_u32(L.b + s * BH * kRowBytes), &tmB, fb, 0,
                           kb * g.N + w.tb * BN + static_cast<int>(rank) * BH);
      };
      auto load_act = [&](int s, int kb, const Unit &w, uint32_t fb) {
        if (SW)
          tma_load_2d_pair(smem_u32(L.b + s * BH * kRowBytes), &tmB, fb, kb * kElemsPerRow,
                           w.tb * BN + static_cast<int>(rank) * BH);
        else
          tma_load_2d_pair(smem_u32(L.a + s * 128 * kRowBytes), &tmA, fb, kb * kElemsPerRow,
                           w.ta * 256 + static_cast<int>(rank) * 128);
      };
      // this CTA's part of its first weight tile goes into the ring (the next
      // k-blocks into the L2) before waiting for the activation pass
      int pre = 0;
      if (pair < P.units) {
        const PairUnit pu = pair_unit(P, pair);
        const Unit w = decode_unit(pu.tile, P.tiles_b, 1);
        pre = g.late_weights ? 0 : min(STAGES, pu.kb1 - pu.kb0);
        for (int i = 0; i < pre; ++i) {
          const uint32_t fb_local = smem_u32(&L.full[i]);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * kStageBytes);
          load_weight(i, pu.kb0 + i, w, mapa_shared(fb_local, 0));
        }
        constexpr int kWRows = SW ? 128 : BH;  // weight rows this CTA loads per k-block
        const int kb2 = min(pu.kb1, pu.kb0 + kPrefetchBytes / (kWRows * kRowBytes));
        for (int kb = pu.kb0 + pre; kb < kb2; ++kb) {
          if (SW)
            tma_prefetch_l2_2d(&tmA, 0, kb * g.N + w.ta * 256 + static_cast<int>(rank) * 128);
          else
            tma_prefetch_l2_2d(&tmB, 0, kb * g.N + w.tb * BN + static_cast<int>(rank) * BH);
        }
      }
      grid_dependency_wait();
      int s = 0;
      uint32_t ph = 0;
      int last_phase[STAGES];
#pragma unroll
      for (int i = 0; i < STAGES; ++i) last_phase[i] = i < pre ? 0 : -1;
      bool ok = true;
      bool first = true;
      for (int u = pair; ok && u < P.units; u += npairs, first = false) {
        const PairUnit pu = pair_unit(P, u);
        const Unit w = decode_unit(pu.tile, P.tiles_b, 1);
        for (int kb = pu.kb0; kb < pu.kb1; ++kb) {
          if (!wait(smem_u32(&L.empty[s]), ph ^ 1u, kWatchProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = smem_u32(&L.full[s]);
          const bool weight_done = first && kb - pu.kb0 < pre;
          if (leader && !weight_done) mbar_arrive_expect_tx(fb_local, 2 * kStageBytes);
          const uint32_t fb = mapa_shared(fb_local, 0);
          load_act(s, kb, w, fb);
          if (!weight_done) load_weight(s, kb, w, fb);
          last_phase[s] = static_cast<int>(ph);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // the leader's full barriers count both CTAs' bytes: once they have
      // completed, no copy is still landing in either CTA
      if (leader)
        for (int i = 0; i < STAGES; ++i)
          if (last_phase[i] >= 0)
            wait(smem_u32(&L.full[i]), static_cast<uint32_t>(last_phase[i]), kWatchProducer);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      grid_dependency_wait();  // bounded waits start once the operands can exist
      // This thread shares its SM sub-partition with four epilogue warps whose
      // arithmetic competes for issue: per k-block it only waits for the
      // stage, advances two precomputed descriptors by a constant and issues
      // the four MMAs as one block.
      int s = 0;
      uint32_t ph = 0;
      uint32_t iter = 0;
      bool ok = true;
      const uint64_t a_desc0 = umma_desc_sw128(smem_u32(L.a)), b_desc0 = umma_desc_sw128(smem_u32(L.b));
      constexpr uint64_t kAStep = (128 * kRowBytes) >> 4, kBStep = (BH * kRowBytes) >> 4;  // per stage
      uint64_t da = a_desc0, db = b_desc0;
      const uint32_t full0 = smem_u32(&L.full[0]), empty0 = smem_u32(&L.empty[0]);
      for (int u = pair; ok && u < P.units; u += npairs, ++iter) {
        const uint32_t buf = iter & 1u;
        const uint32_t acc_ph = (iter >> 1) & 1u;
        if (!wait(smem_u32(&L.tempty[buf]), acc_ph ^ 1u, kWatchMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        const PairUnit pu = pair_unit(P, u);
        for (int kb = pu.kb0; kb < pu.kb1; ++kb) {
          if (!wait(full0 + 8u * s, ph, kWatchMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          umma_pair_kblock<KIND == Kind::I8>(d_tmem, da, db, kIdesc, kb > pu.kb0 ? 1u : 0u);
          tc_commit_pair_mc(empty0 + 8u * s, 0x3);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
            da = a_desc0;
            db = b_desc0;
          } else {
            da += kAStep;
            db += kBStep;
          }
        }
        if (ok) tc_commit_pair_mc(smem_u32(&L.tfull[buf]), 0x3);
      }
      tc_commit_pair(smem_u32(L.mma_done));
      wait(smem_u32(L.mma_done), 0, kWatchMma);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    EpiCtx c;
    c.g = &g;
    c.P = &P;
    c.tmOut = &tmOut;
    c.L = L;
    c.q = warp & 3;
    c.part = (warp - 2) / 4;
    c.lane = lane;
    c.epi_t = threadIdx.x - 64;
    c.scr = L.scratch + (warp - 2) * kWarpScratch;
    c.prm = L.params + (warp - 2) * kWarpParams;
    const bool has_bias = g.bias != nullptr;
    grid_dependency_wait();  // row scales come from the activation pass
    if constexpr (SW) {
      epilogue_loop_sw_dispatch<KIND, BN>(g, P, L, c.prm, tmem_base, c.q, c.part, lane, pair, npairs, rank,
                                          peer_abort);
    } else {
      uint32_t iter = 0;
      for (int u = pair; u < P.units; u += npairs, ++iter) {
        c.w = decode_unit(u, P.tiles_b, 1);
        const uint32_t buf = iter & 1u;
        c.full_bar = smem_u32(&L.tfull[buf]);
        c.full_parity = (iter >> 1) & 1u;
        c.row0 = c.w.ta * 256 + static_cast<int>(rank) * 128;
        c.t_row = tmem_base + (static_cast<uint32_t>(c.q * 32) << 16) + buf * BN;
        c.empty_bar = mapa_shared(smem_u32(&L.tempty[buf]), 0);
        c.empty_remote = true;
        // the epilogue hands the buffer back to the leader once its TMEM reads are done
        const bool ok = epilogue_dispatch<KIND, BN, false>(c, g.mode, has_bias);
        if (!ok) st_shared_cluster(peer_abort, 1u);
      }
      if (lane == 0) bulk_wait_all();
    }
  }

  // the leader's MMAs (which read both CTAs' shared memory) are complete and
  // every TMEM read is done before either CTA releases TMEM or exits
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TCOLS);
  }
}

// --------------------------------------------------------------- planning
// 0: INT8 shapes with M <= 16 run the register-fed decode kernel (decode.cu);
// 1: they run the swapped tcgen05 kernel like 16 < M <= 32.
std::atomic<int> g_decode_kernel{0};

// Tile plan keyed on M:
//  * I8, M <= 16 and (M <= 8 or a K-split swapped plan): the register-fed
//    decode kernel (decode.cu): weights stream from HBM into registers and
//    warp MMAs, in (column group, k-block) ranges balanced over the SMs.
//  * I8 and M <= 32: swapped orientation (weights fill the 128-row MMA
//    dimension, the activation rows are the MMA N = 16 or 32); the K range is
//    split over CTAs until the grid covers the SMs, with an exact INT32
//    reduction.  These shapes stream the weight once and are HBM-bound.
//  * large M: CTA-pair tiles of 256 rows x BN in {256, 128}, whichever needs
//    less time over the SM pairs: tile rounds (wave quantisation) x the cost
//    of one round of that width (kPairCost*), as long as the tiles fill at
//    least half of the pairs.
//  * otherwise: activation rows in 128-row tiles and the widest weight tile
//    N in {256, 128, 64, 32} that still gives one CTA per SM.
//  In the normal orientation K stays whole inside a CTA (no split), so the
//  FP16 accumulation order never depends on the plan.
// Relative time of one CTA-pair tile wave by tile width: a 256 x 128 tile
// does half the work of a 256 x 256 tile but its N = 128 pair MMAs issue at
// about 0.72 of the N = 256 rate (C4 measured 1.38x slower with 128-wide
// tiles), so it costs 128 / 0.72 ~ 178 against 256.
constexpr long long kPairCost256 = 256, kPairCost128 = 178;

GemmPlan plan_gemm(Kind kind, int M, int N, int K, int num_sms) {
  GemmPlan p;
  p.kind = kind;
  const int elems = kind == Kind::I8 ? 128 : 64;
  p.kb_total = (K + elems - 1) / elems;
  const int pairs = num_sms / 2;
  if (M > 128) {
    const long long u256 = static_cast<long long>((M + 255) / 256) * ((N + 255) / 256);
    const long long u128 = static_cast<long long>((M + 255) / 256) * ((N + 127) / 128);
    if (u128 * 2 >= pairs) {
      const long long cost256 = (u256 + pairs - 1) / pairs * kPairCost256;
      const long long cost128 = (u128 + pairs - 1) / pairs * kPairCost128;
      p.pair = true;
      p.bn = cost256 <= cost128 ? 256 : 128;
      p.tiles_a = (M + 255) / 256;
      p.tiles_b = (N + p.bn - 1) / p.bn;
      p.splits = 1;
      p.kb_per_split = p.kb_total;
      p.units = p.tiles_a * p.tiles_b;
      p.grid = 2 * (p.units < pairs ? p.units : pairs);
      p.smem = smem2_bytes_for(p.bn);
      return p;
    }
  }
  if (kind == Kind::I8 && M <= 32) {
    p.swap = true;
    p.bn = M <= 16 ? 16 : 32;
    p.tiles_a = (N + 127) / 128;
    p.tiles_b = (M + p.bn - 1) / p.bn;
    int splits = num_sms / (p.tiles_a * p.tiles_b);
    splits = splits < 1 ? 1 : splits;
    const int max_splits = p.kb_total / 8 > 0 ? p.kb_total / 8 : 1;
    splits = splits > max_splits ? max_splits : splits;
    p.kb_per_split = (p.kb_total + splits - 1) / splits;
    p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
    // The register-fed kernel streams faster where the swapped plan splits K
    // (its INT32 partials meet in HBM) and at M <= 8 (one MMA per k-step);
    // with 16 rows and whole-K tiles the tcgen05 kernel is faster.
    if (M <= 16 && N % 16 == 0 && g_decode_kernel.load() == 0 && (M <= 8 || p.splits > 1)) {
      plan_decode_i8(p, M, N, K, num_sms);
      return p;
    }
  } else {
    p.swap = false;
    p.tiles_a = (M + 127) / 128;
    const int cands[4] = {256, 128, 64, 32};
    p.bn = 32;
    for (int c : cands) {
      // accept one wave that leaves at most ~15% of the SMs idle
      if (static_cast<long long>(p.tiles_a) * ((N + c - 1) / c) * 20 >= 17LL * num_sms) {
        p.bn = c;
        break;
      }
    }
    p.tiles_b = (N + p.bn - 1) / p.bn;
    p.splits = 1;
    p.kb_per_split = p.kb_total;
  }
  p.units = p.tiles_a * p.tiles_b * p.splits;
  p.grid = p.units < num_sms ? p.units : num_sms;
  p.smem = smem_bytes_for(p.bn, p.swap);
  return p;
}

// The swapped orientation of a CTA-pair plan: 256-column weight tiles (the
// pair's MMA M) by BN-row activation tiles (MMA N), BN in {256, 128} by the
// same wave cost as the normal orientation.  Its epilogue stores from
// registers, which serves row-major outputs (modes 0-2 and the raw mode 4) of
// one destination; the channel-major store (mode 3), the plane export (mode 5)
// and the multi-destination run keep the normal orientation.
std::atomic<int> g_pair_direct{1};

bool pair_sw_eligible(const GemmPlan &p, int mode, int n_outs) {
  return p.pair && p.kind == Kind::I8 && n_outs == 1 && (mode == 0 || mode == 1 || mode == 2 || mode == 4) &&
         g_pair_direct.load() != 0;
}

GemmPlan plan_pair_sw(const GemmPlan &normal, int M, int N, int num_sms) {
  GemmPlan p = normal;
  const int pairs = num_sms / 2;
  const long long tw = (N + 255) / 256;
  const long long u256 = tw * ((M + 255) / 256), u128 = tw * ((M + 127) / 128);
  const long long cost256 = (u256 + pairs - 1) / pairs * kPairCost256;
  const long long cost128 = (u128 + pairs - 1) / pairs * kPairCost128;
  p.pair_sw = true;
  p.bn = cost256 <= cost128 ? 256 : 128;
  p.tiles_a = static_cast<int>(tw);
  p.tiles_b = (M + p.bn - 1) / p.bn;
  p.units = p.tiles_a * p.tiles_b;
  p.full_units = p.units;
  p.tail_s = 1;
  p.grid = 2 * (p.units < pairs ? p.units : pairs);
  p.smem = smem2_bytes_for(p.bn, true);
  return p;
}

// Tail split of a swapped pair plan.  With T tiles on P pairs the last round
// holds T mod P tiles and leaves the other pairs idle for a whole tile time.
// When that round is at most half full, its tiles are cut into S = P / (T mod
// P) pieces of consecutive k-blocks (at least kTailMinKb each), one per pair,
// so the round takes about 1/S of a tile plus the exchange of the pieces'
// INT32 sums (each piece stores the (S-1)/S of the tile it does not own,
// waits for the others and finishes its own rows: ~4 us).  Measured on the
// C3 shapes: fc2 (48 k-blocks per tile) gains; 12-k-block tiles (out
// projection, fc1) lose, hence kTailMinTileKb.
constexpr int kTailMinKb = 4, kTailMinTileKb = 24;
std::atomic<int> g_pair_tail{1};

static void split_tail(GemmPlan &p, int num_sms) {
  const int pairs = num_sms / 2;
  const int tail = p.units % pairs;
  if (g_pair_tail.load() == 0 || tail == 0 || p.kb_total < kTailMinTileKb) return;
  int pieces = pairs / tail;
  if (pieces > p.kb_total / kTailMinKb) pieces = p.kb_total / kTailMinKb;
  if (pieces > p.bn / 32) pieces = p.bn / 32;  // every piece owns a 32-row chunk
  if (pieces < 2) return;
  p.full_units = p.units - tail;
  p.tail_s = pieces;
  p.units = p.full_units + tail * pieces;
  p.grid = 2 * (p.units < pairs ? p.units : pairs);
}

GemmPlan plan_for(Kind kind, int M, int N, int K, int num_sms, int mode, int n_outs, bool tail_split) {
  const GemmPlan p = plan_gemm(kind, M, N, K, num_sms);
  if (!pair_sw_eligible(p, mode, n_outs)) return p;
  GemmPlan q = plan_pair_sw(p, M, N, num_sms);
  if (tail_split) split_tail(q, num_sms);
  return q;
}

size_t splitk_ws_bytes(const GemmPlan &p) {
  if (p.reg) return decode_ws_bytes(p);
  return p.splits > 1 ? static_cast<size_t>(p.tiles_a) * p.tiles_b * 128 * p.bn * 4 : 0;
}
size_t splitk_count_bytes(const GemmPlan &p) {
  if (p.reg) return static_cast<size_t>(p.tiles_a) * 4;
  if (p.tail_s > 1) return static_cast<size_t>(p.units - p.full_units) * 2 * 4;  // per tail tile, piece, CTA
  return p.splits > 1 ? static_cast<size_t>(p.tiles_a) * p.tiles_b * 4 : 0;
}
size_t tail_slot_bytes(const GemmPlan &p) {
  if (p.tail_s < 2) return 0;
  return static_cast<size_t>(p.units - p.full_units) * 2 * static_cast<size_t>(p.bn) * 128 * 4;
}

// GEMM launch with programmatic stream serialisation: its prologue (barriers,
// TMEM, descriptor and L2 weight prefetch) overlaps the activation pass.
template <typename Fn>
static cudaError_t launch_dependent(Fn fn, int grid, size_t smem, cudaStream_t st, const CUtensorMap &tmA,
                                    const CUtensorMap &tmB, const OutMaps &tmOut, const KernelParams &P) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, tmA, tmB, tmOut, P);
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <Kind KIND, int BN, bool SWAP>
static cudaError_t launch_one(const GemmPlan &p, const CUtensorMap &tmA, const CUtensorMap &tmB,
                              const OutMaps &tmOut, const GemmArgs &a, cudaStream_t st) {
  auto fn = gemm_kernel<KIND, BN, SWAP>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = smem_bytes_for(BN, SWAP);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  KernelParams P;
  P.a = a;
  P.tiles_a = p.tiles_a;
  P.tiles_b = p.tiles_b;
  P.splits = p.splits;
  P.kb_total = p.kb_total;
  P.kb_per_split = p.kb_per_split;
  P.units = p.units;
  return counted(launch_dependent(fn, p.grid, smem, st, tmA, tmB, tmOut, P));
}

template <Kind KIND, int BN, bool SW>
static cudaError_t launch_pair(const GemmPlan &p, const CUtensorMap &tmA, const CUtensorMap &tmB,
                               const OutMaps &tmOut, const GemmArgs &a, cudaStream_t st) {
  auto fn = gemm2_kernel<KIND, BN, SW>;
  static bool configured[64] = {};  // per instantiation and device
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = smem2_bytes_for(BN, SW);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  KernelParams P;
  P.a = a;
  P.tiles_a = p.tiles_a;
  P.tiles_b = p.tiles_b;
  P.splits = 1;
  P.kb_total = p.kb_total;
  P.kb_per_split = p.kb_total;
  P.units = p.units;
  P.tail_s = SW && p.tail_s > 1 ? p.tail_s : 1;
  P.full_units = P.tail_s > 1 ? p.full_units : p.units;
  // grid is a multiple of the pair (cluster dimensions are compiled in)
  return counted(launch_dependent(fn, p.grid, smem, st, tmA, tmB, tmOut, P));
}

cudaError_t launch_gemm(const GemmPlan &p, const CUtensorMap &tmA, const CUtensorMap &tmB,
                        const OutMaps &tmOut, const GemmArgs &a, cudaStream_t st) {
  if (p.reg) return launch_decode_i8(p, a, st);
  if (p.pair) {
    if (p.grid % 2) return cudaErrorInvalidConfiguration;
    if (p.kind == Kind::I8) {
      if (p.pair_sw) {
        if (p.bn == 256) return launch_pair<Kind::I8, 256, true>(p, tmA, tmB, tmOut, a, st);
        if (p.bn == 128) return launch_pair<Kind::I8, 128, true>(p, tmA, tmB, tmOut, a, st);
      } else {
        if (p.bn == 256) return launch_pair<Kind::I8, 256, false>(p, tmA, tmB, tmOut, a, st);
        if (p.bn == 128) return launch_pair<Kind::I8, 128, false>(p, tmA, tmB, tmOut, a, st);
      }
    } else if (!p.pair_sw) {
      if (p.bn == 256) return launch_pair<Kind::F16, 256, false>(p, tmA, tmB, tmOut, a, st);
      if (p.bn == 128) return launch_pair<Kind::F16, 128, false>(p, tmA, tmB, tmOut, a, st);
    }
    return cudaErrorInvalidConfiguration;
  }
  if (p.kind == Kind::I8) {
    if (p.swap) {
      if (p.bn == 16) return launch_one<Kind::I8, 16, true>(p, tmA, tmB, tmOut, a, st);
      if (p.bn == 32) return launch_one<Kind::I8, 32, true>(p, tmA, tmB, tmOut, a, st);
    } else {
      switch (p.bn) {
        case 256: return launch_one<Kind::I8, 256, false>(p, tmA, tmB, tmOut, a, st);
        case 128: return launch_one<Kind::I8, 128, false>(p, tmA, tmB, tmOut, a, st);
        case 64: return launch_one<Kind::I8, 64, false>(p, tmA, tmB, tmOut, a, st);
        case 32: return launch_one<Kind::I8, 32, false>(p, tmA, tmB, tmOut, a, st);
        default: break;
      }
    }
  } else if (!p.swap) {
    switch (p.bn) {
      case 256: return launch_one<Kind::F16, 256, false>(p, tmA, tmB, tmOut, a, st);
      case 128: return launch_one<Kind::F16, 128, false>(p, tmA, tmB, tmOut, a, st);
      case 64: return launch_one<Kind::F16, 64, false>(p, tmA, tmB, tmOut, a, st);
      case 32: return launch_one<Kind::F16, 32, false>(p, tmA, tmB, tmOut, a, st);
      default: break;
    }
  }
  return cudaErrorInvalidConfiguration;
}

}  // namespace htpg
