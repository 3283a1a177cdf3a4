// Opcodes 2-4 of the reference (HTP_OPS_MAT_MUL_PERMUTED_W4D16A32 /
// W8D16A32 / W4D16A32_IQ4_NL): FP32 activations times a weight stored as
// ggml blocks (Q4_0, Q8_0, IQ4_NL), dequantised to FP16 and accumulated in
// FP32 (reference: mat_mul.c:246-430 dequantisation, :1601-1874 GEMM;
// quants.h:11-31 block layouts).
//
//  * dq_chunk            one 16-byte row chunk (8 consecutive k of one column)
//                        of the FP16 weight from a super-block, in registers
//  * qk0_dequant_kernel  whole weight -> FP16 rows (the large-M path feeds the
//                        FP16 GEMM with it; also the standalone dequantiser)
//  * qk0_repack_kernel   one-time reorder of the super-blocks into per-stage
//                        records (cached per weight like the other repacks)
//  * qgemm_swap_kernel   small M: one bulk copy per stage streams the
//                        super-block record, dequantiser warps write the
//                        FP16 weight tile into shared memory in the 128-byte
//                        swizzled K-major layout, one thread issues
//                        tcgen05.mma with that tile as the 128-row operand and
//                        the FP16 activations as the narrow one; iterations
//                        (tile, k-block) are split evenly over the CTAs
//                        (stream-K) and partial tiles are summed in a fixed
//                        order by the last CTA to finish them.
#include <cuda_fp16.h>

#include "kernels.h"
#include "ptx.cuh"

namespace htpg {

// ================================================================ decode
// IQ4_NL levels (the reference's iq4_nl_to_fp16_lut, mat_mul.c:34-37), stored
// as level + 128 so that 0x64 | byte is the FP16 number 1024 + level + 128.
constexpr int kIq4Levels[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
constexpr uint32_t iq4_word(int i) {
  return static_cast<uint32_t>(kIq4Levels[i] + 128) | static_cast<uint32_t>(kIq4Levels[i + 1] + 128) << 8 |
         static_cast<uint32_t>(kIq4Levels[i + 2] + 128) << 16 | static_cast<uint32_t>(kIq4Levels[i + 3] + 128) << 24;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) { return __byte_perm(a, b, sel); }
// Packed FP16 arithmetic with explicit round-to-nearest (never contracted).
__device__ __forceinline__ uint32_t hsub2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2_rn(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Bytes level+128 of the four nibbles in bits [0, 16) of x: two 8-entry byte
// tables selected by the nibbles' low three bits, merged by their fourth bit.
// prmt.b32 in its default mode, where a selector nibble with bit 3 set gives
// the selected byte's sign bit replicated (__byte_perm ignores that bit).
__device__ __forceinline__ uint32_t prmt_sx(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t iq4_lookup4(uint32_t x) {
  // nibbles >= 8 give sign bytes in lo; the select below takes hi for them
  const uint32_t lo = prmt_sx(iq4_word(0), iq4_word(4), x);
  const uint32_t hi = prmt_sx(iq4_word(8), iq4_word(12), x & 0x7777u);
  // 0xFF where the nibble is >= 8: bit 3 of nibble 1 / 3 is the sign bit of
  // byte 0 / 1 of x, that of nibble 0 / 2 the sign bit of byte 0 / 1 of x << 4
  const uint32_t msk = prmt_sx(x, x << 4, 0x9D8Cu);
  return (hi & msk) | (lo & ~msk);
}

// FP16 elements k = 8j .. 8j+7 (of the tile's 32) of column m (of the tile's
// 32) from super-block j of a 32 x 32 tile.  Element e of a super-block is the
// packed-FP16 offset e (see kernels.h), so these eight elements are
// e = {0,1, 64,65, 128,129, 192,193} + 2m: the pairs (k, k+1) belong to the
// reference's output vectors v = 0..3 and use scale 2v + m/16.
//  Q8_0:        code = byte e.
//  Q4_0/IQ4_NL: code = low (v < 2) or high nibble of byte 2*(e%64) + (v&1),
//               i.e. of the four bytes b0..b3 at 4m: k order b0.lo, b2.lo,
//               b1.lo, b3.lo, b0.hi, b2.hi, b1.hi, b3.hi (mat_mul.c:389-424).
// Codes become exact FP16 integers by the magic-number method (0x64XX is the
// FP16 number 1024 + XX, minus 1024 + offset), then one packed multiply with
// the scale rounds code * scale to nearest: the FP16 value the reference's
// qf16 multiply and conversion produce (mat_mul.c:420-423, 521-524).
// The raw words of one chunk: the super-block's scale vector and the codes
// (Q4_0/IQ4_NL: the word at 4m; Q8_0: the four byte pairs at 2m + 64v).
struct ChunkWords {
  uint4 sc;
  uint32_t q[4];
};
template <int QT>
__device__ __forceinline__ ChunkWords chunk_words_global(const uint8_t *blk, int m) {
  ChunkWords w;
  w.sc = ld_dep(reinterpret_cast<const uint4 *>(blk));
  if constexpr (QT == kGgmlQ8_0) {
#pragma unroll
    for (int v = 0; v < 4; ++v) w.q[v] = ld_dep(reinterpret_cast<const uint16_t *>(blk + 16 + 2 * m + 64 * v));
  } else {
    w.q[0] = ld_dep(reinterpret_cast<const uint32_t *>(blk + 16 + 4 * m));
  }
  return w;
}
template <int QT>
__device__ __forceinline__ ChunkWords chunk_words_shared(uint32_t blk, int m) {
  ChunkWords w;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(w.sc.x), "=r"(w.sc.y), "=r"(w.sc.z), "=r"(w.sc.w)
               : "r"(blk));
  if constexpr (QT == kGgmlQ8_0) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      uint16_t h;
      asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(blk + 16 + 2 * m + 64 * v));
      w.q[v] = h;
    }
  } else {
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w.q[0]) : "r"(blk + 16 + 4 * m));
  }
  return w;
}

template <int QT>
__device__ __forceinline__ uint4 dq_decode(const ChunkWords &cw, int m) {
  const uint4 sc = cw.sc;
  const uint32_t ssel = (m & 16) ? 0x3232u : 0x1010u;  // broadcast scale 2v + (m >= 16)
  const uint32_t s0 = prmt(sc.x, sc.x, ssel), s1 = prmt(sc.y, sc.y, ssel);
  const uint32_t s2 = prmt(sc.z, sc.z, ssel), s3 = prmt(sc.w, sc.w, ssel);
  uint32_t h0, h1, h2, h3, bias;
  if constexpr (QT == kGgmlQ8_0) {
    // [code_k, 0x64, code_k+1, 0x64], sign bit flipped: 1024 + code + 128
    h0 = prmt(cw.q[0], 0x64646464u, 0x5140u) ^ 0x00800080u;
    h1 = prmt(cw.q[1], 0x64646464u, 0x5140u) ^ 0x00800080u;
    h2 = prmt(cw.q[2], 0x64646464u, 0x5140u) ^ 0x00800080u;
    h3 = prmt(cw.q[3], 0x64646464u, 0x5140u) ^ 0x00800080u;
    bias = 0x64806480u;  // 1152
  } else {
    const uint32_t w = cw.q[0];
    if constexpr (QT == kGgmlQ4_0) {
      h0 = (w & 0x000F000Fu) | 0x64006400u;          // b0.lo, b2.lo
      h1 = ((w >> 8) & 0x000F000Fu) | 0x64006400u;   // b1.lo, b3.lo
      h2 = ((w >> 4) & 0x000F000Fu) | 0x64006400u;   // b0.hi, b2.hi
      h3 = ((w >> 12) & 0x000F000Fu) | 0x64006400u;  // b1.hi, b3.hi
      bias = 0x64086408u;                            // 1032: nibble - 8
    } else {
      const uint32_t ra = iq4_lookup4(w);        // b0.lo b0.hi b1.lo b1.hi
      const uint32_t rb = iq4_lookup4(w >> 16);  // b2.lo b2.hi b3.lo b3.hi
      h0 = (prmt(ra, rb, 0x0400u) & 0x00FF00FFu) | 0x64006400u;
      h1 = (prmt(ra, rb, 0x0602u) & 0x00FF00FFu) | 0x64006400u;
      h2 = (prmt(ra, rb, 0x0501u) & 0x00FF00FFu) | 0x64006400u;
      h3 = (prmt(ra, rb, 0x0703u) & 0x00FF00FFu) | 0x64006400u;
      bias = 0x64806480u;  // 1152
    }
  }
  return make_uint4(hmul2_rn(hsub2_rn(h0, bias), s0), hmul2_rn(hsub2_rn(h1, bias), s1),
                    hmul2_rn(hsub2_rn(h2, bias), s2), hmul2_rn(hsub2_rn(h3, bias), s3));
}

// ============================================================ dequantiser
// A warp per (32-column tile, 64-deep k-block); lane = column.  Each lane
// writes the 128 bytes of its column's k-block (eight chunks); the reads of a
// chunk step are 32 consecutive words of one super-block.  REC: the source is
// the stage records (zero-padded past K and N) instead of the stream.
template <int QT, bool REC>
__global__ void __launch_bounds__(256) qk0_dequant_kernel(uint16_t *__restrict__ dst, const uint8_t *__restrict__ src,
                                                          int k, int n, long long stride_kb, long long stride_n) {
  grid_dependents_launch();
  grid_dependency_wait();  // the weight may come from the kernel before this one
  constexpr int BLK = QT == kGgmlQ8_0 ? 272 : 144;
  const int ntiles = n / 32, ktiles = k / 32;
  const long long wid = static_cast<long long>(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  const int kb_total = (ktiles + 1) / 2;
  if (wid >= static_cast<long long>(ntiles) * kb_total) return;
  const int nt = static_cast<int>(wid % ntiles), kb = static_cast<int>(wid / ntiles);
  uint16_t *row = dst + kb * stride_kb + static_cast<long long>(nt * 32 + lane) * stride_n;
  // record (nt/4, kb) holds this tile's eight super-blocks at ((nt%4)*2 + c/4)*4 + c%4
  const uint8_t *rec = src + ((static_cast<size_t>(nt / 4) * kb_total + kb) * 32 + (nt % 4) * 8) * BLK;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int kt = 2 * kb + c / 4;
    if (REC || kt < ktiles) {
      const uint8_t *blk = REC ? rec + c * BLK : src + ((static_cast<size_t>(nt) * ktiles + kt) * 4 + (c & 3)) * BLK;
      *reinterpret_cast<uint4 *>(row + c * 8) = dq_decode<QT>(chunk_words_global<QT>(blk, lane), lane);
    }
  }
}

cudaError_t launch_qk0_dequant(uint16_t *dst, const uint8_t *src, int qt, int k, int n, long long stride_kb,
                               long long stride_n, bool records, cudaStream_t st) {
  const long long warps = static_cast<long long>(n / 32) * ((k / 32 + 1) / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((warps + 7) / 8), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
#define HTPG_QK0_DQ(T)                                                                                  \
  (records ? cudaLaunchKernelEx(&cfg, qk0_dequant_kernel<T, true>, dst, src, k, n, stride_kb, stride_n) \
           : cudaLaunchKernelEx(&cfg, qk0_dequant_kernel<T, false>, dst, src, k, n, stride_kb, stride_n))
  if (qt == kGgmlQ4_0)
    e = HTPG_QK0_DQ(kGgmlQ4_0);
  else if (qt == kGgmlQ8_0)
    e = HTPG_QK0_DQ(kGgmlQ8_0);
  else if (qt == kGgmlIQ4_NL)
    e = HTPG_QK0_DQ(kGgmlIQ4_NL);
  else
    return cudaErrorInvalidValue;
#undef HTPG_QK0_DQ
  return counted(e != cudaSuccess ? e : cudaGetLastError());
}

// ================================================================ repack
// Stage records for the fused kernel: record (ta, kb) holds, contiguously and
// in this order, the super-blocks of column tiles 4ta..4ta+3, k-tiles 2kb and
// 2kb+1 (tile r, k-tile e, super-block j at ((r*2 + e)*4 + j) blocks), with
// zeros for tiles past N or K.  Records are ordered (ta, kb), so one
// pipeline stage is one contiguous copy.  One thread per 16 bytes.
__global__ void __launch_bounds__(256) qk0_repack_kernel(uint4 *__restrict__ dst, const uint4 *__restrict__ src,
                                                         int blk16, int ktiles, int ntiles, int kb_total,
                                                         long long units) {
  const long long u = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u >= units) return;
  const int per_rec = 32 * blk16;  // 16-byte units per record
  const long long rec = u / per_rec;
  const int w = static_cast<int>(u % per_rec);
  const int sb = w / blk16, part = w % blk16;  // super-block of the record, unit within it
  const int r = sb >> 3, e = (sb >> 2) & 1, j = sb & 3;
  const int ta = static_cast<int>(rec / kb_total), kb = static_cast<int>(rec % kb_total);
  const int nt = 4 * ta + r, kt = 2 * kb + e;
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (nt < ntiles && kt < ktiles)
    v = ld_dep(src + ((static_cast<long long>(nt) * ktiles + kt) * 4 + j) * blk16 + part);
  dst[u] = v;
}

size_t qk0_stage_records_bytes(int qt, int k, int n) {
  const size_t recs = static_cast<size_t>((n + 127) / 128) * static_cast<size_t>((k / 32 + 1) / 2);
  return recs * 32u * static_cast<size_t>(qk0_block_bytes(qt));
}

cudaError_t launch_qk0_repack(uint8_t *dst, const uint8_t *src, int qt, int k, int n, cudaStream_t st) {
  const int blk16 = qk0_block_bytes(qt) / 16;
  if (!blk16) return cudaErrorInvalidValue;
  const int ktiles = k / 32, ntiles = n / 32, kb_total = (ktiles + 1) / 2;
  const long long units = static_cast<long long>(qk0_stage_records_bytes(qt, k, n) / 16u);
  qk0_repack_kernel<<<static_cast<unsigned>((units + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<uint4 *>(dst), reinterpret_cast<const uint4 *>(src), blk16, ktiles, ntiles, kb_total, units);
  return counted(cudaGetLastError());
}

// ============================================================ fused GEMM
// Dequantisers: kQGroups groups of four warps; group g converts the CTA's
// iterations g, g + kQGroups, ...; warp r of a group (r = warp % 4, its TMEM
// lane quadrant) converts the 32 rows of column tile r, eight independent
// chunks per lane.
//
// The MMA issuer commits once per kCommit iterations: a tcgen05.commit costs
// about as much as a dozen N=16 MMAs on this part, so the FP16 operand ring is
// released kCommit slots at a time (one commit barrier per half of the ring).
// The activation tile of an iteration (BN rows x 64 k) lives with its operand
// slot: the converting group's 128 threads read it from the FP32 activations
// (one 8-element chunk each, 16 rows; two for 32) and round it to FP16, so no
// copy-engine request sits behind the super-block prefetch and no separate
// conversion kernel runs.  The super-block ring is released by the
// dequantisers alone.
constexpr int kQGroups = 4;
constexpr int kQDeqWarps = 4 * kQGroups;
constexpr int kQEpiWarps = 4;   // one per TMEM lane quadrant
constexpr int kQThreads = 32 * (2 + kQEpiWarps + kQDeqWarps);
constexpr int kCommit = 4;              // iterations per MMA commit
constexpr int kAStages = 2 * kCommit;  // FP16 operand ring (dequantisers -> MMA)
constexpr int kQMaxStages = 24;         // super-block ring (bulk copies -> dequantisers)
constexpr int kQSmemLimit = 232448;
constexpr int kQBarBytes = 1024;
static_assert(kQGroups == kCommit, "each commit group holds one iteration of every dequantiser group");

__host__ __device__ constexpr int q_block_bytes(int qt) { return qt == kGgmlQ8_0 ? 272 : 144; }
// one stage: 4 column tiles x 2 k-tiles x 4 super-blocks (128 columns x 64 k)
__host__ __device__ constexpr int q_stage_bytes(int qt) { return 32 * q_block_bytes(qt); }
__host__ __device__ constexpr int q_stages(int qt, int bn) {
  return (kQSmemLimit - 1024 - kQBarBytes - kAStages * (16384 + bn * 128)) / q_stage_bytes(qt) < kQMaxStages
             ? (kQSmemLimit - 1024 - kQBarBytes - kAStages * (16384 + bn * 128)) / q_stage_bytes(qt)
             : kQMaxStages;
}
__host__ __device__ constexpr size_t qgemm_smem(int qt, int bn) {
  return 1024 + static_cast<size_t>(kAStages) * (16384 + bn * 128) +
         static_cast<size_t>(q_stages(qt, bn)) * q_stage_bytes(qt) + kQBarBytes;
}
static_assert((2 * kQMaxStages + kAStages + 7) * 8 + 16 <= kQBarBytes, "barrier block");
static_assert(kQGroups <= q_stages(kGgmlQ8_0, 32), "super-block slots advance by kQGroups");
static_assert(qgemm_smem(kGgmlQ8_0, 32) <= kQSmemLimit && qgemm_smem(kGgmlQ4_0, 32) <= kQSmemLimit,
              "shared memory budget");

struct QGemmParams {
  QGemmArgs a;
  const uint8_t *w;  // stage records (qk0_repack_kernel)
  int tiles_b, kb_total;
  long long iters;
};

// Stream-K bookkeeping: CTA c owns iterations [c*T/G, (c+1)*T/G).
__device__ __forceinline__ int sk_owner(long long i, long long T, int G) {
  return static_cast<int>(((i + 1) * G - 1) / T);
}
__device__ __forceinline__ long long sk_begin(int c, long long T, int G) { return static_cast<long long>(c) * T / G; }
// Partial slot of CTA c's piece of tile t: slot 0 for its first tile, slot 1
// for its last (only these two can be partial).
__device__ __forceinline__ int sk_slot(int c, int t, long long T, int G, int KB) {
  return 2 * c + (t == static_cast<int>(sk_begin(c, T, G) / KB) ? 0 : 1);
}

template <int BN>
__device__ __forceinline__ void qgemm_store(const QGemmArgs &g, const float (&v)[BN], int n, int tb) {
  if (n >= g.N) return;
#pragma unroll
  for (int j = 0; j < BN; ++j) {
    const int m = tb * BN + j;
    if (m < g.M) g.out[static_cast<long long>(m) * g.ldo + n] = v[j];
  }
}

template <int QT, int BN>
__global__ void __launch_bounds__(kQThreads, 1)
    qgemm_swap_kernel(const QGemmParams P) {
  constexpr int QS = q_stages(QT, BN);
  constexpr uint32_t QSB = q_stage_bytes(QT);
  constexpr uint32_t BB = BN * 128;
  constexpr int BLK = q_block_bytes(QT);
  constexpr uint32_t TCOLS = 2 * BN <= 32 ? 32 : 64;
  constexpr uint32_t kIdesc = idesc_f16(128, BN);
  static_assert(BN == 16 || BN == 32, "activation rows per tile");
  static_assert(BN * 8 % 128 == 0, "activation chunks per group thread");

  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *sA = base;                    // kAStages x 128 rows x 128 B (FP16 weight, swizzled)
  uint8_t *sB = sA + kAStages * 16384;   // kAStages x BN rows x 128 B (FP16 activations, swizzled)
  uint8_t *sQ = sB + kAStages * BB;      // QS x one stage record
  uint64_t *bars = reinterpret_cast<uint64_t *>(sQ + QS * QSB);
  uint64_t *qfull = bars, *qempty = qfull + QS;
  uint64_t *afull = qempty + QS;
  uint64_t *mdone = afull + kAStages;    // [2]: the MMAs of a commit group have completed
  uint64_t *tfull = mdone + 2, *tempty = tfull + 2, *mma_done = tempty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
  volatile uint32_t *flag = tmem_slot + 1;
  volatile uint32_t *abort = tmem_slot + 2;

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const QGemmArgs &g = P.a;
  uint32_t *wd = g.watchdog;
  grid_dependents_launch();

  if (threadIdx.x == 0) {
    for (int s = 0; s < QS; ++s) {
      mbar_init(smem_u32(&qfull[s]), 1);
      mbar_init(smem_u32(&qempty[s]), 4);  // the converting group's four warps
    }
    for (int s = 0; s < kAStages; ++s) mbar_init(smem_u32(&afull[s]), 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&mdone[b]), 1);
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), kQEpiWarps);
    }
    mbar_init(smem_u32(mma_done), 1);
    *abort = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TCOLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const long long T = P.iters;
  const int G = gridDim.x, cta = blockIdx.x, KB = P.kb_total;
  const long long i0 = sk_begin(cta, T, G), i1 = sk_begin(cta + 1, T, G);

  if (warp == 0) {
    // ------------------------------------------------ super-block producer
    if (lane == 0) {
      // (tile, k-block) of the first iteration; later ones by incrementing
      // (a 64-bit division per iteration would cost more than the iteration)
      const int t0 = static_cast<int>(i0 / KB), kb0 = static_cast<int>(i0 % KB);
      // stage record of iteration (ta, kb): one contiguous run of QSB bytes
      auto record = [&](int ta, int kb) { return P.w + (static_cast<size_t>(ta) * KB + kb) * QSB; };
      // warm the L2 with the first records; loads wait for the previous kernel
      {
        int ta = t0 / P.tiles_b, tb = t0 % P.tiles_b, kb = kb0;
        for (long long i = i0; i < i1 && i < i0 + QS; ++i) {
          bulk_prefetch_l2(record(ta, kb), QSB);
          if (++kb == KB) {
            kb = 0;
            if (++tb == P.tiles_b) tb = 0, ++ta;
          }
        }
      }
      grid_dependency_wait();
      int s = 0;
      uint32_t ph = 0;
      int last_phase[QS];
#pragma unroll
      for (int j = 0; j < QS; ++j) last_phase[j] = -1;
      int ta = t0 / P.tiles_b, tb = t0 % P.tiles_b, kb = kb0;
      for (long long i = i0; i < i1; ++i) {
        if (!mbar_wait(smem_u32(&qempty[s]), ph ^ 1u, wd, kWatchProducer, abort)) break;
        const uint32_t fb = smem_u32(&qfull[s]);
        mbar_arrive_expect_tx(fb, QSB);
        bulk_load(smem_u32(sQ + s * QSB), record(ta, kb), QSB, fb);
        if (++kb == KB) {
          kb = 0;
          if (++tb == P.tiles_b) tb = 0, ++ta;
        }
        last_phase[s] = static_cast<int>(ph);
        if (++s == QS) {
          s = 0;
          ph ^= 1u;
        }
      }
      // no copy may still be landing when the CTA exits
      for (int j = 0; j < QS; ++j)
        if (last_phase[j] >= 0)
          mbar_wait(smem_u32(&qfull[j]), static_cast<uint32_t>(last_phase[j]), wd, kWatchProducer, abort);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    // Iterations go in commit groups of kCommit, split where a new accumulator
    // piece starts (its buffer may only be waited for once every earlier
    // piece's completion has been committed): every wait of a run first, then
    // its MMAs back to back; one commit per group frees its operand slots.
    if (lane == 0) {
      grid_dependency_wait();
      bool ok = true;
      uint32_t piece = 0;  // accumulator pieces (tiles or tile parts) finished
      int kb_g = static_cast<int>(i0 % KB);
      for (long long i = i0; ok && i < i1;) {
        const long long j = i - i0;
        const long long gend = i0 + (j / kCommit + 1) * kCommit < i1 ? i0 + (j / kCommit + 1) * kCommit : i1;
        // the run [i, send): up to the group's end or the next piece start
        long long send = i + 1;
        for (int kb = kb_g + 1 == KB ? 0 : kb_g + 1; send < gend && kb != 0; kb = kb + 1 == KB ? 0 : kb + 1) ++send;
        if (i == i0 || kb_g == 0)
          ok = mbar_wait(smem_u32(&tempty[piece & 1u]), ((piece >> 1) & 1u) ^ 1u, wd, kWatchMma, abort);
        for (long long t = i; ok && t < send; ++t) {
          const int sa = static_cast<int>((t - i0) % kAStages);
          const uint32_t aph = static_cast<uint32_t>(((t - i0) / kAStages) & 1);
          ok = mbar_wait(smem_u32(&afull[sa]), aph, wd, kWatchMma, abort);
        }
        if (!ok) break;
        tc_fence_after();
        for (long long t = i; t < send; ++t, kb_g = kb_g + 1 == KB ? 0 : kb_g + 1) {
          const int sa = static_cast<int>((t - i0) % kAStages);
          const uint32_t buf = piece & 1u;
          umma_f16_kblock(tmem_base + buf * BN, umma_desc_sw128(smem_u32(sA + sa * 16384)),
                          umma_desc_sw128(smem_u32(sB + sa * BB)), kIdesc, (t == i0 || kb_g == 0) ? 0u : 1u);
          if (t == i1 - 1 || kb_g == KB - 1) {
            tc_commit(smem_u32(&tfull[buf]));
            ++piece;
          }
        }
        if (send == gend && (gend - i0) % kCommit == 0) tc_commit(smem_u32(&mdone[(j / kCommit) & 1]));
        i = send;
      }
      // every MMA of this thread completes before TMEM is released
      tc_commit(smem_u32(mma_done));
      mbar_wait(smem_u32(mma_done), 0, wd, kWatchMma, abort);
    }
  } else if (warp < 2 + kQEpiWarps) {
    // ------------------------------------------------ epilogue (one warp per lane quadrant)
    const int q = warp & 3;
    const bool lead = threadIdx.x == 64;
    grid_dependency_wait();  // nothing is stored before the previous kernel is done
    uint32_t piece = 0;
    for (long long i = i0; i < i1; ++piece) {
      const int t = static_cast<int>(i / KB);
      const long long tile_end = static_cast<long long>(t + 1) * KB;
      const long long end = i1 < tile_end ? i1 : tile_end;
      const bool whole = (i % KB) == 0 && end == tile_end;
      const uint32_t buf = piece & 1u;
      const bool ok = mbar_wait(smem_u32(&tfull[buf]), (piece >> 1) & 1u, wd, kWatchEpilogue, abort);
      tc_fence_after();
      float v[BN];
#pragma unroll
      for (int j = 0; j < BN; ++j) v[j] = 0.0f;
      if (ok) {
        const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
        if constexpr (BN == 16) {
          uint32_t r[16];
          tmem_ld16(taddr, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
        } else {
          uint32_t r[32];
          tmem_ld32(taddr, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && ok) mbar_arrive(smem_u32(&tempty[buf]));
      const int tb = t % P.tiles_b;
      const int n = (t / P.tiles_b) * 128 + q * 32 + lane;
      if (whole) {
        if (ok) qgemm_store<BN>(g, v, n, tb);
      } else {
        // partial tile: park it, count it; the last contributor sums all
        // contributions in CTA order (deterministic) and stores the tile
        float *mine = g.partials + static_cast<size_t>(sk_slot(cta, t, T, G, KB)) * BN * 128 + q * 32 + lane;
#pragma unroll
        for (int j = 0; j < BN; ++j) mine[j * 128] = v[j];
        __threadfence();
        named_bar_sync(1, 32 * kQEpiWarps);
        const int c_first = sk_owner(static_cast<long long>(t) * KB, T, G);
        const int c_last = sk_owner(tile_end - 1, T, G);
        if (lead) {
          uint32_t fin = 0u;
          if (!*abort) {
            const uint32_t prev = atomicAdd(g.counters + t, 1u);
            fin = prev == static_cast<uint32_t>(c_last - c_first) ? 1u : 0u;
          }
          *flag = fin;
        }
        named_bar_sync(1, 32 * kQEpiWarps);
        if (*flag) {
          __threadfence();
          float acc[BN];
#pragma unroll
          for (int j = 0; j < BN; ++j) acc[j] = 0.0f;
          for (int cc = c_first; cc <= c_last; ++cc) {
            const float *p = g.partials + static_cast<size_t>(sk_slot(cc, t, T, G, KB)) * BN * 128 + q * 32 + lane;
#pragma unroll
            for (int j = 0; j < BN; ++j) acc[j] += __ldcg(p + j * 128);
          }
          qgemm_store<BN>(g, acc, n, tb);
          if (lead) g.counters[t] = 0u;
        }
        named_bar_sync(1, 32 * kQEpiWarps);  // the flag is reused by the next piece
      }
      i = end;
    }
  } else {
    // ------------------------------------------------ dequantisers
    const int dw = warp - 2 - kQEpiWarps;
    const int grp = dw >> 2, nt = warp & 3;  // group; column tile = this warp's lane quadrant
    const int gt = nt * 32 + lane;  // thread of the group: activation chunks gt, gt + 128, ...
    grid_dependency_wait();  // the activations come from the kernel before this one
    const uint32_t sQs = smem_u32(sQ), sAs = smem_u32(sA), sBs = smem_u32(sB);
    const int row = nt * 32 + lane;
    const uint32_t row_off = static_cast<uint32_t>(row) * 128u;
    // ring slots and phases of iteration j = grp, grp + kQGroups, ...
    int sq = grp;
    uint32_t qph = 0;
    int tb = 0, kb = 0;
    {
      const long long ig = i0 + grp;
      if (ig < i1) tb = static_cast<int>((ig / KB) % P.tiles_b), kb = static_cast<int>(ig % KB);
    }
    for (long long i = i0 + grp; i < i1; i += kQGroups) {
      const long long j = i - i0;
      const int sa = static_cast<int>(j % kAStages);
      // the operand slot is free once the MMAs of iteration j - kAStages completed
      const uint32_t md_par = static_cast<uint32_t>(((j / kAStages) & 1) ^ 1);
      // activation chunks of this iteration: FP32 loads issued before the waits
      constexpr int kChunks = BN * 8 / 128;
      float4 xa[kChunks][2];
#pragma unroll
      for (int u = 0; u < kChunks; ++u) {
        const int q = gt + 128 * u, r = q >> 3, c = q & 7;
        const int m = tb * BN + r, k0 = kb * 64 + c * 8;
        if (m < g.M && k0 < g.K) {
          const float4 *src = reinterpret_cast<const float4 *>(g.x + static_cast<long long>(m) * g.K + k0);
          xa[u][0] = ld_dep(src);  // written by the kernel before this one
          xa[u][1] = ld_dep(src + 1);
        } else {
          xa[u][0] = xa[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      bool ok = mbar_wait(smem_u32(&mdone[(j / kCommit) & 1]), md_par, wd, kWatchDequant, abort);
      ok = ok && mbar_wait(smem_u32(&qfull[sq]), qph, wd, kWatchDequant, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      const uint32_t qs = sQs + sq * QSB + nt * 8 * BLK;  // this column tile's 2 k-tiles x 4 super-blocks
      const uint32_t as = sAs + sa * 16384 + row_off;
      ChunkWords cw[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) cw[c] = chunk_words_shared<QT>(qs + c * BLK, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&qempty[sq]));  // the record has been read
      // the activation tile (FP16, round to nearest even, like the reference's
      // conversion mat_mul.c:114-148), 128-byte swizzled
#pragma unroll
      for (int u = 0; u < kChunks; ++u) {
        const int q = gt + 128 * u, r = q >> 3, c = q & 7;
        const float f[8] = {xa[u][0].x, xa[u][0].y, xa[u][0].z, xa[u][0].w,
                            xa[u][1].x, xa[u][1].y, xa[u][1].z, xa[u][1].w};
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          h[e] = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(f[2 * e]))) |
                 static_cast<uint32_t>(__half_as_ushort(__float2half_rn(f[2 * e + 1]))) << 16;
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(sBs + sa * BB + r * 128 + ((c ^ (r & 7)) << 4)),
                     "r"(h[0]), "r"(h[1]), "r"(h[2]), "r"(h[3])
                     : "memory");
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 val = dq_decode<QT>(cw[c], lane);
        // 128-byte swizzle: chunk c of row r at position c ^ (r % 8)
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(as + ((c ^ (row & 7)) << 4)),
                     "r"(val.x), "r"(val.y), "r"(val.z), "r"(val.w)
                     : "memory");
      }
      fence_proxy_async_smem();  // the MMA (async proxy) reads what this thread wrote
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&afull[sa]));
      if ((sq += kQGroups) >= QS) sq -= QS, qph ^= 1u;
      for (kb += kQGroups; kb >= KB;) {
        kb -= KB;
        if (++tb == P.tiles_b) tb = 0;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TCOLS);
  }
}

// ============================================= register-fed decode (M <= 32)
// Each CTA owns NW (16, 8 or 4) 32-column weight tiles and one range of
// 32-deep k-tiles; 16 / NW warps share a tile, each a part of the range, and
// add their FP32 sums in shared memory in a fixed order.  It first rounds its
// slice of x to FP16 into shared memory (the reference's activation rounding).
// Each warp streams its tile's super-blocks from the stage records into its
// own shared-memory ring with cp.async (a k-tile pair of one tile is 8
// consecutive super-blocks, 1152 or 2176 bytes; four pairs in flight), decodes
// only the FP16 pairs its MMA fragments hold, with dq_decode's arithmetic, and
// accumulates with mma.sync m16n8k16 (FP16 x FP16 -> FP32), NT = 1, 2 or 4
// 8-token MMA tiles (M <= 8, 16, 32).  Fragment layout:
// lane (g, t) holds tile columns 4g .. 4g+3 (MMA rows g / g+8 of column group
// cg are columns 4g + 2cg / 4g + 2cg + 1, so a lane's codes of one super-block
// are adjacent in shared memory), pair t of super-blocks 2s and 2s+1 (k = 16s
// + 2t, +1 and 16s + 8 + 2t, +1 of the tile's 32); the activation fragment
// holds the same k.  The k ranges' FP32 partial tiles meet in a workspace
// (lane-major: each lane's values in one 128-byte row per element); the last
// range to arrive sums them in range order (deterministic) and writes the
// output.  No thread waits for another CTA.
constexpr int kQdWarps = 16, kQdThreads = 32 * kQdWarps;
constexpr int kQdStages = 4;       // k-tile pairs of a warp's tile in flight
constexpr int kQdMaxSplits = 32;   // k ranges per tile at most (the last one sums them all)
__host__ __device__ constexpr int qd_pair_bytes(int qt) { return 8 * (qt == kGgmlQ8_0 ? 272 : 144); }

struct QDecParams {
  const uint8_t *w;   // stage records
  const float *x;     // [M][K]
  float *out;         // [M][ldo]
  float *part;        // [ntiles][S][32 columns][16 tokens]
  uint32_t *cnt;      // [ntiles], zero before the launch, left zero
  int M, N, K, ldo;
  int ntiles, ktiles, kb_total, S, pitch;  // pitch: halves per activation row in shared memory
  int nw;                                  // weight tiles per CTA (16 / nw warps per tile)
};

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The raw words one lane needs from one 32 x 32 tile (four super-blocks) in
// shared memory: scale word t of each super-block and the codes of columns
// 4g .. 4g+3 (Q4_0 / IQ4_NL: the columns' code words, one 16-byte load per
// super-block; Q8_0: pair t of the four columns, one 8-byte load, two columns
// per word: q[j][0] = q[j][1] and q[j][2] = q[j][3]).
struct QdWords {
  uint32_t sc[4];
  uint32_t q[4][4];  // [super-block][column 4g + c]
};

// Plain loads (the compiler may schedule them; the ring's cp.async wait,
// which clobbers memory, keeps them after the stage has landed).
template <int QT>
__device__ __forceinline__ void qd_load(QdWords &w, const uint8_t *tile, int g, int t) {
  constexpr int BLK = QT == kGgmlQ8_0 ? 272 : 144;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint8_t *sb = tile + j * BLK;
    w.sc[j] = *reinterpret_cast<const uint32_t *>(sb + 4 * t);
    if constexpr (QT == kGgmlQ8_0) {
      const uint2 q = *reinterpret_cast<const uint2 *>(sb + 16 + 8 * g + 64 * t);
      w.q[j][0] = w.q[j][1] = q.x;
      w.q[j][2] = w.q[j][3] = q.y;
    } else {
      const uint4 q = *reinterpret_cast<const uint4 *>(sb + 16 + 16 * g);
      w.q[j][0] = q.x;
      w.q[j][1] = q.y;
      w.q[j][2] = q.z;
      w.q[j][3] = q.w;
    }
  }
}

// Pair t (k = 2t, 2t+1 of the super-block's eight) of one column: the same
// operations as dq_decode's element pair t.  s: the column's scale (scale
// 2v + column / 16 of the super-block's eight) in both halves.  sh = 4 * the
// nibble index of the pair's first code in the word: dq_decode's pairs are
// (b0.lo, b2.lo), (b1.lo, b3.lo), (b0.hi, b2.hi), (b1.hi, b3.hi), i.e.
// nibbles 0, 2, 1, 3 and the same + 4 (computed without branches:
// ((t & 1) << 3) | ((t >> 1) << 2)).  Q8_0: HI takes the word's upper pair.
template <int QT, bool HI>
__device__ __forceinline__ uint32_t qd_pair(uint32_t s, uint32_t q, int sh) {
  uint32_t h, bias;
  if constexpr (QT == kGgmlQ8_0) {
    h = prmt(q, 0x64646464u, HI ? 0x5342u : 0x5140u) ^ 0x00800080u;
    bias = 0x64806480u;
  } else if constexpr (QT == kGgmlQ4_0) {
    h = ((q >> sh) & 0x000F000Fu) | 0x64006400u;
    bias = 0x64086408u;
  } else {
    // the pair's two nibbles looked up together, levels into the two halves
    const uint32_t y = ((q >> sh) & 0xFu) | (((q >> (sh + 16)) & 0xFu) << 4);
    h = prmt(iq4_lookup4(y), 0u, 0x5140u) | 0x64006400u;
    bias = 0x64806480u;
  }
  return hmul2_rn(hsub2_rn(h, bias), s);
}

// Pair t of one column in two super-blocks (words q0, q1 with broadcast
// scales s0, s1): qd_pair twice.  IQ4_NL looks the four nibbles up together: one
// byte permute gathers bytes (t & 1) and (t & 1) + 2 of both words, the shift
// by s4 = 4 * (t >> 1) brings the pair's nibbles to the bytes' low halves,
// and x = A0 | A1 << 4 | B0 << 8 | B1 << 12 indexes the table (A, B: the
// pair's nibbles at sh and sh + 16 of q0 and q1).
template <int QT, bool HI>
__device__ __forceinline__ void qd_pair2(uint32_t s0, uint32_t s1, uint32_t q0, uint32_t q1, int sh, uint32_t gsel,
                                         int s4, uint32_t &r0, uint32_t &r1) {
  if constexpr (QT == kGgmlIQ4_NL) {
    const uint32_t w = prmt(q0, q1, gsel) >> s4;
    const uint32_t lv = iq4_lookup4((w & 0x0F0Fu) | ((w >> 12) & 0xF0F0u));  // L(A0) L(A1) L(B0) L(B1)
    const uint32_t bias = 0x64806480u;
    r0 = hmul2_rn(hsub2_rn(prmt(lv, 0x64646464u, 0x4240u), bias), s0);
    r1 = hmul2_rn(hsub2_rn(prmt(lv, 0x64646464u, 0x4341u), bias), s1);
  } else {
    r0 = qd_pair<QT, HI>(s0, q0, sh);
    r1 = qd_pair<QT, HI>(s1, q1, sh);
  }
}

// Position of word w of an activation row in the shared-memory slice: each
// 16-k group (8 words) holds its pairs in the order 0, 4, 1, 5, 2, 6, 3, 7,
// so that a lane's two activation words (pairs t and t + 4) are one 8-byte load.
__device__ __forceinline__ int qd_xpos(int w) { return (w & ~7) | ((w & 3) << 1) | ((w >> 2) & 1); }

__device__ __forceinline__ uint32_t f2_to_h2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// MB: the CTAs per SM the launch bounds promise (a plan for two CTAs per SM
// keeps 64 registers per thread; one CTA per SM may use up to 128).
template <int QT, int NT, int MB>
__global__ void __launch_bounds__(kQdThreads, MB) qdec_kernel(const QDecParams P) {
  constexpr int BLK = QT == kGgmlQ8_0 ? 272 : 144;
  constexpr int TILEF = 256 * NT;  // floats of one partial tile: 32 columns x 8 NT tokens
  constexpr int PAIR = qd_pair_bytes(QT);
  extern __shared__ __align__(16) uint32_t qd_smem[];  // [16 warps][stages][PAIR] rings, then the x slice
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int sh = ((t & 1) << 3) | ((t >> 1) << 2);  // see qd_pair
  const uint32_t gsel = 0x6420u + 0x1111u * static_cast<uint32_t>(t & 1);  // see qd_pair2
  const int s4 = (t >> 1) << 2;
  const uint32_t ssel = g >= 4 ? 0x3232u : 0x1010u;  // columns 4g.. >= 16: the upper scale of each pair
  const int grp = blockIdx.x / P.S, sp = blockIdx.x - grp * P.S;
  const int kt0 = static_cast<int>(static_cast<long long>(P.ktiles) * sp / P.S);
  const int kt1 = static_cast<int>(static_cast<long long>(P.ktiles) * (sp + 1) / P.S);
  const int kw_parts = kQdWarps / P.nw, ks = warp / P.nw;  // this warp's part of the range
  const int nt = grp * P.nw + (warp - ks * P.nw);
  const int wk0 = kt0 + (kt1 - kt0) * ks / kw_parts, wk1 = kt0 + (kt1 - kt0) * (ks + 1) / kw_parts;
  const bool active = nt < P.ntiles && wk1 > wk0;
  const uint32_t ring = smem_u32(qd_smem) + static_cast<uint32_t>(warp * kQdStages * PAIR);
  uint32_t *qd_x = qd_smem + kQdWarps * kQdStages * PAIR / 4;  // [8 NT rows][pitch / 2] f16x2, see qd_xpos
  // k-tile pair pp (k-tiles 2pp, 2pp+1) of this warp's tile: 8 consecutive
  // super-blocks of record (nt/4, pp), starting at block (nt%4)*8
  const int pp0 = wk0 >> 1, npairs = active ? ((wk1 - 1) >> 1) - pp0 + 1 : 0;
  // this lane's first 16-byte chunk of pair pp0; records of one tile group are 32 * BLK apart
  const uint8_t *wsrc = P.w + (static_cast<size_t>(nt >> 2) * P.kb_total + pp0) * (32u * BLK) +
                        static_cast<size_t>((nt & 3) << 3) * BLK + 16 * lane;
  auto issue_pair = [&](int i) {  // pair pp0 + i into stage i % stages (one commit group per call)
    if (active && i < npairs) {
      const uint8_t *src = wsrc + static_cast<size_t>(i) * (32u * BLK);
      const uint32_t dst = ring + static_cast<uint32_t>((i % kQdStages) * PAIR) + 16 * lane;
#pragma unroll
      for (int c = 0; c < (PAIR / 16 + 31) / 32; ++c)
        if (lane + 32 * c < PAIR / 16)
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + 512 * c), "l"(src + 512 * c) : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  grid_dependents_launch();
  // the weight is prepared once (static): its first pairs stream now
#pragma unroll
  for (int i = 0; i < kQdStages; ++i) issue_pair(i);
  grid_dependency_wait();  // x may be the previous operator's output
  // this CTA's slice of x, rounded to FP16 (rows >= M are zero)
  const int kw = (kt1 - kt0) * 32;  // k per row of the slice
  for (int i = threadIdx.x; i < 8 * NT * (kw / 4); i += kQdThreads) {
    const int r = i / (kw / 4), c4 = i - r * (kw / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < P.M) v = ld_dep(reinterpret_cast<const float4 *>(P.x + static_cast<size_t>(r) * P.K + kt0 * 32) + c4);
    qd_x[r * (P.pitch / 2) + qd_xpos(2 * c4)] = f2_to_h2(v.x, v.y);
    qd_x[r * (P.pitch / 2) + qd_xpos(2 * c4 + 1)] = f2_to_h2(v.z, v.w);
  }
  __syncthreads();

  float acc[2][NT][4];
#pragma unroll
  for (int cg = 0; cg < 2; ++cg)
#pragma unroll
    for (int jt = 0; jt < NT; ++jt)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[cg][jt][r] = 0.0f;
  for (int i = 0; i < npairs; ++i) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kQdStages - 1) : "memory");  // pair i has landed
    __syncwarp();
    const uint8_t *stage = reinterpret_cast<const uint8_t *>(qd_smem) + (warp * kQdStages + i % kQdStages) * PAIR;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int kt = 2 * (pp0 + i) + e;
      if (kt < wk0 || kt >= wk1) continue;
      QdWords cur;
      qd_load<QT>(cur, stage + e * 4 * BLK, g, t);
      const int kl = (kt - kt0) * 32;  // k of the tile within the slice
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2) {
        uint32_t b[NT][2];
#pragma unroll
        for (int jt = 0; jt < NT; ++jt) {
          // pairs t and t + 4 of the 16-k group: adjacent words (qd_xpos)
          const uint2 bv = *reinterpret_cast<const uint2 *>(qd_x + (8 * jt + g) * (P.pitch / 2) + (kl + 16 * s2) / 2 + 2 * t);
          b[jt][0] = bv.x;
          b[jt][1] = bv.y;
        }
        // the lane's column scales of the two super-blocks, both halves
        const uint32_t sl = prmt(cur.sc[2 * s2], cur.sc[2 * s2], ssel);
        const uint32_t su = prmt(cur.sc[2 * s2 + 1], cur.sc[2 * s2 + 1], ssel);
#pragma unroll
        for (int cg = 0; cg < 2; ++cg) {
          const int c0 = 2 * cg, c1 = 2 * cg + 1;
          uint32_t a0, a1, a2, a3;
          qd_pair2<QT, false>(sl, su, cur.q[2 * s2][c0], cur.q[2 * s2 + 1][c0], sh, gsel, s4, a0, a2);
          qd_pair2<QT, true>(sl, su, cur.q[2 * s2][c1], cur.q[2 * s2 + 1][c1], sh, gsel, s4, a1, a3);
#pragma unroll
          for (int jt = 0; jt < NT; ++jt) mma_f16_16816(acc[cg][jt], a0, a1, a2, a3, b[jt][0], b[jt][1]);
        }
      }
    }
    __syncwarp();  // every lane is done with the stage before it is refilled
    issue_pair(i + kQdStages);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  // accumulator element (cg, jt, r) of this lane in a partial tile (32
  // columns x 8 NT tokens): lane-major, so that a warp's stores and loads of
  // one element are 128 bytes
  auto elem = [&](int cg, int jt, int r) { return ((cg * NT + jt) * 4 + r) * 32 + lane; };
  if (kw_parts > 1) {
    // the tile's warps add their parts in part order, through shared memory
    // (over the rings, which every warp has finished with)
    float *red = reinterpret_cast<float *>(qd_smem);  // [part][nw][TILEF]
    __syncthreads();
    if (nt < P.ntiles)
#pragma unroll
      for (int cg = 0; cg < 2; ++cg)
#pragma unroll
        for (int jt = 0; jt < NT; ++jt)
#pragma unroll
          for (int r = 0; r < 4; ++r) red[(ks * P.nw + (warp - ks * P.nw)) * TILEF + elem(cg, jt, r)] = acc[cg][jt][r];
    __syncthreads();
    if (ks != 0 || nt >= P.ntiles) return;
#pragma unroll
    for (int cg = 0; cg < 2; ++cg)
#pragma unroll
      for (int jt = 0; jt < NT; ++jt)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float v = red[warp * TILEF + elem(cg, jt, r)];
          for (int q = 1; q < kw_parts; ++q) v = __fadd_rn(v, red[(q * P.nw + warp) * TILEF + elem(cg, jt, r)]);
          acc[cg][jt][r] = v;
        }
  } else if (nt >= P.ntiles) {
    return;
  }
  // this range's partial tile, then the arrival; the last range of the tile
  // sums all ranges' partials in range order and writes the output
  float *mine = P.part + (static_cast<size_t>(nt) * P.S + sp) * TILEF;
#pragma unroll
  for (int cg = 0; cg < 2; ++cg)
#pragma unroll
    for (int jt = 0; jt < NT; ++jt)
#pragma unroll
      for (int r = 0; r < 4; ++r) mine[elem(cg, jt, r)] = acc[cg][jt][r];
  __syncwarp();
  uint32_t prev = 0u;
  if (lane == 0)
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(P.cnt + nt) : "memory");
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev != static_cast<uint32_t>(P.S - 1)) return;
  __syncwarp();  // lane 0's acquire orders every lane's reads below
  const float *all = P.part + static_cast<size_t>(nt) * P.S * TILEF;
  // the lane's elements of every range: QB ranges' loads in flight at a time,
  // added in range order
  // (with up to 128 registers per thread twice as many as with 64)
  constexpr int QB = (MB == 1 ? 8 : 4) / NT;
#pragma unroll
  for (int cg = 0; cg < 2; ++cg)
#pragma unroll
    for (int jt = 0; jt < NT; ++jt)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[cg][jt][r] = 0.0f;
  for (int q0 = 0; q0 < P.S; q0 += QB) {
    float u[QB][2][NT][4];
#pragma unroll
    for (int qq = 0; qq < QB; ++qq)
#pragma unroll
      for (int cg = 0; cg < 2; ++cg)
#pragma unroll
        for (int jt = 0; jt < NT; ++jt)
#pragma unroll
          for (int r = 0; r < 4; ++r)
            u[qq][cg][jt][r] = q0 + qq < P.S ? __ldcg(all + (q0 + qq) * TILEF + elem(cg, jt, r)) : 0.0f;
#pragma unroll
    for (int qq = 0; qq < QB; ++qq)
      if (q0 + qq < P.S) {
#pragma unroll
        for (int cg = 0; cg < 2; ++cg)
#pragma unroll
          for (int jt = 0; jt < NT; ++jt)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[cg][jt][r] = __fadd_rn(acc[cg][jt][r], u[qq][cg][jt][r]);
      }
  }
#pragma unroll
  for (int cg = 0; cg < 2; ++cg)
#pragma unroll
    for (int jt = 0; jt < NT; ++jt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int col = 4 * g + 2 * cg + (r >> 1), tok = 8 * jt + 2 * t + (r & 1);
        if (tok < P.M) P.out[static_cast<size_t>(tok) * P.ldo + nt * 32 + col] = acc[cg][jt][r];
      }
  if (lane == 0) P.cnt[nt] = 0u;
}

std::atomic<int> g_qdec{1};
std::atomic<int> g_qdec_shape{0};

// Candidates: one or two CTAs per SM (two where both CTAs' rings and slices
// fit in the SM's shared memory) x 16, 8 or 4 weight tiles per CTA (narrower
// groups put 2 or 4 warps on each tile).  Each takes as many k ranges as fill
// its CTA slots, at least as many as make the widest range's FP16 slice fit
// beside the rings, at most kQdMaxSplits and two k-tiles per warp.  The
// estimate of a candidate: 8 us per wave of CTAs (the fixed part of a CTA's
// life: slice load, ring fill, hand-off; a second wave costs it again), the
// busiest SM's streaming work (CTAs spread over the SMs first: ceil(grid /
// SMs) x tiles x k-tiles of a range, in k-tile units of this type's bytes at
// an SM's share of the HBM bandwidth), the finishing warp's L2 round trips
// (ceil(S / QB) batches of partial loads) and, where warps share a tile, the
// sum of their parts in shared memory (one round trip's worth per extra part
// and 8-token tile).  The smallest estimate wins; ties keep one CTA per SM
// (fewer CTAs) and wider groups.  On the LLM projections (K x N = 4096 x 14336
// and 14336 x 4096, m = 1..32, every type) it picks the fastest measured
// shape or one within 4%.
QDecPlan plan_qdec(int qt, int M, int N, int K, int num_sms) {
  QDecPlan best;
  best.grid = 0;
  const int nt = M <= 8 ? 1 : M <= 16 ? 2 : 4;
  const int ntiles = N / 32, ktiles = K / 32;
  const size_t rings = static_cast<size_t>(kQdWarps) * kQdStages * qd_pair_bytes(qt);
  // one k-tile of one 32-column tile: four super-blocks; 13 ns per 576 bytes
  // at ~44 GB/s per SM, against ~700 ns per dependent L2 round trip
  const double kt_ns = 4.0 * (qt == kGgmlQ8_0 ? 272 : 144) / 44.0, trip_ns = 700.0, wave_ns = 8000.0;
  const int force = g_qdec_shape.load();
  double best_cost = 0.0;
  // rows 8 words apart in the banks (16 halves of padding): a half-warp's
  // 8-byte activation loads (4 rows x 32 bytes) hit every bank once
  auto slice_bytes = [&](int S) { return static_cast<size_t>(8 * nt) * ((ktiles + S - 1) / S * 32 + 16) * 2; };
  for (int per_sm = 1; per_sm <= 2; ++per_sm) {
    // per CTA: 113 KB of the SM's 228 (1 KB of each CTA's is reserved) with
    // two; the kernel's launch bounds keep two CTAs' registers within the SM's
    const size_t budget = per_sm == 2 ? 112 * 1024 : 227 * 1024;
    if (rings >= budget) continue;
    const size_t slice_max = budget - rings < kQdMaxSlice ? budget - rings : kQdMaxSlice;
    const int target = per_sm * num_sms;
    const int qb = (per_sm == 1 ? 8 : 4) / nt;  // the finisher's ranges per batch (qdec_kernel's QB)
    for (int nw = kQdWarps; nw >= 4; nw /= 2) {
      if (force && force != per_sm * 100 + nw) continue;
      const int groups = (ntiles + nw - 1) / nw, parts = kQdWarps / nw;
      int s_max = ktiles / (2 * parts);
      s_max = s_max < 1 ? 1 : s_max > kQdMaxSplits ? kQdMaxSplits : s_max;
      int S = target / groups;
      S = S < 1 ? 1 : S > s_max ? s_max : S;
      while (slice_bytes(S) > slice_max && S < ktiles) ++S;
      if (slice_bytes(S) > slice_max) continue;
      const long long grid = static_cast<long long>(groups) * S;
      const long long busiest = (grid + num_sms - 1) / num_sms, waves = (grid + target - 1) / target;
      const double cost = static_cast<double>(waves) * wave_ns +
                          static_cast<double>(busiest) * nw * ((ktiles + S - 1) / S) * kt_ns +
                          static_cast<double>((S + qb - 1) / qb) * trip_ns +
                          static_cast<double>((parts - 1) * nt) * trip_ns;
      if (best.grid == 0 || cost < best_cost) {
        best_cost = cost;
        best.nt = nt;
        best.ntiles = ntiles;
        best.ktiles = ktiles;
        best.nw = nw;
        best.per_sm = per_sm;
        best.splits = S;
        best.grid = static_cast<int>(grid);
        best.pitch = (ktiles + S - 1) / S * 32 + 16;  // halves
        best.smem = slice_bytes(S);                  // the slice (the rings are added per type)
      }
    }
  }
  return best;  // grid 0: no candidate (a forced shape that does not fit)
}
size_t qdec_smem_bytes(int qt, const QDecPlan &p) {
  const size_t s = static_cast<size_t>(kQdWarps) * kQdStages * qd_pair_bytes(qt) + p.smem;
  // a plan sized for one CTA per SM asks for more than half the SM's shared
  // memory, so that its CTAs spread over the SMs instead of pairing up on
  // some of them while others stay empty
  return p.per_sm == 1 && s < 116 * 1024 ? 116 * 1024 : s;
}

template <int QT, int NT, int MB>
static cudaError_t launch_qdec_t(const QDecPlan &p, const uint8_t *w, const QGemmArgs &a, cudaStream_t st) {
  auto fn = qdec_kernel<QT, NT, MB>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const size_t smem = qdec_smem_bytes(QT, p);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    // all of the SM's unified memory as shared memory: two CTAs' rings fit
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  QDecParams P;
  P.w = w;
  P.x = a.x;
  P.out = a.out;
  P.part = a.partials;
  P.cnt = a.counters;
  P.M = a.M;
  P.N = a.N;
  P.K = a.K;
  P.ldo = static_cast<int>(a.ldo);
  P.ntiles = p.ntiles;
  P.ktiles = p.ktiles;
  P.kb_total = (a.K + 63) / 64;
  P.S = p.splits;
  P.pitch = p.pitch;
  P.nw = p.nw;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
  cfg.blockDim = dim3(kQdThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, P);
  return counted(e != cudaSuccess ? e : cudaGetLastError());
}

cudaError_t launch_qdec(int qt, const QDecPlan &p, const uint8_t *w, const QGemmArgs &a, cudaStream_t st) {
  if (a.M < 1 || a.M > 32 || a.N % 32 || a.K % 32 || p.smem > kQdMaxSlice) return cudaErrorInvalidConfiguration;
#define HTPG_QDEC_NT(T, MB)                                                 \
  (p.nt == 1   ? launch_qdec_t<T, 1, MB>(p, w, a, st)                       \
   : p.nt == 2 ? launch_qdec_t<T, 2, MB>(p, w, a, st)                       \
               : launch_qdec_t<T, 4, MB>(p, w, a, st))
#define HTPG_QDEC(T) (p.per_sm == 1 ? HTPG_QDEC_NT(T, 1) : HTPG_QDEC_NT(T, 2))
  if (qt == kGgmlQ4_0) return HTPG_QDEC(kGgmlQ4_0);
  if (qt == kGgmlQ8_0) return HTPG_QDEC(kGgmlQ8_0);
  if (qt == kGgmlIQ4_NL) return HTPG_QDEC(kGgmlIQ4_NL);
#undef HTPG_QDEC
#undef HTPG_QDEC_NT
  return cudaErrorInvalidValue;
}

QGemmPlan plan_qgemm(int qt, int M, int N, int K, int num_sms) {
  QGemmPlan p;
  p.bn = M <= 16 ? 16 : 32;
  p.tiles_a = (N + 127) / 128;
  p.tiles_b = (M + p.bn - 1) / p.bn;
  p.kb_total = (K + 63) / 64;
  p.iters = static_cast<long long>(p.tiles_a) * p.tiles_b * p.kb_total;
  // at least four k-blocks per CTA, at most one CTA per SM
  long long g = p.iters / 4;
  g = g < 1 ? 1 : g;
  p.grid = static_cast<int>(g < num_sms ? g : num_sms);
  p.smem = qgemm_smem(qt, p.bn);
  return p;
}

template <int QT, int BN>
static cudaError_t launch_qgemm_t(const QGemmPlan &p, const uint8_t *w, const QGemmArgs &a, cudaStream_t st) {
  auto fn = qgemm_swap_kernel<QT, BN>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const size_t smem = qgemm_smem(QT, BN);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  QGemmParams P;
  P.a = a;
  P.w = w;
  P.tiles_b = p.tiles_b;
  P.kb_total = p.kb_total;
  P.iters = p.iters;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
  cfg.blockDim = dim3(kQThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, P);
  return counted(e != cudaSuccess ? e : cudaGetLastError());
}

cudaError_t launch_qgemm(int qt, const QGemmPlan &p, const uint8_t *w,
                         const QGemmArgs &a, cudaStream_t st) {
  if (p.grid < 1 || p.iters < p.grid) return cudaErrorInvalidConfiguration;
  if (qt == kGgmlQ4_0) return p.bn == 16 ? launch_qgemm_t<kGgmlQ4_0, 16>(p, w, a, st)
                                         : launch_qgemm_t<kGgmlQ4_0, 32>(p, w, a, st);
  if (qt == kGgmlQ8_0) return p.bn == 16 ? launch_qgemm_t<kGgmlQ8_0, 16>(p, w, a, st)
                                         : launch_qgemm_t<kGgmlQ8_0, 32>(p, w, a, st);
  if (qt == kGgmlIQ4_NL) return p.bn == 16 ? launch_qgemm_t<kGgmlIQ4_NL, 16>(p, w, a, st)
                                           : launch_qgemm_t<kGgmlIQ4_NL, 32>(p, w, a, st);
  return cudaErrorInvalidValue;
}

}  // namespace htpg
