// CTA-pair W8A8 GEMM with the weight tile resident on chip (opcode 15
// arithmetic, linear_w8a8.c:130-192), for K <= 1536.  Not the default: the
// streaming CTA-pair kernel of kernels.cu is faster (htpg_set_tmem_weights).
//
// The CTA-pair kernel of kernels.cu moves both operands through shared memory:
// per SM and 128 x 256 x 32 MMA step, 8 KB of TMA writes and 12 KB of tensor-
// core reads (each CTA's B half is read by both SMs), plus 8 B per output
// element of epilogue staging.  Its time follows those bytes (256- against
// 128-column tiles: 1.38x the time for 1.40x the operand bytes).  Here the
// operands swap roles:
//  * A = the weight: each CTA of the pair keeps its 128 weight columns for as
//    long as it works on them, k-blocks 0..7 in tensor memory (INT8, 4 per
//    32-bit column: lane = weight column, column kb*32 + k/4) and k-blocks
//    8..11 resident in shared memory (loaded by TMA once per tile);
//  * B = the activation codes: 128 tokens per MMA (N = 128), 64 rows per CTA,
//    streamed by TMA through a shared-memory ring of 4 k-blocks per stage;
//  * D = 256 weight columns x 128 tokens, double-buffered in TMEM columns
//    [0, 128) and [128, 256); the weight's TMEM part sits in [256, 512).
// The epilogue needs no staging: TMEM lane = output column, so for each token
// a warp stores 32 consecutive FP32 outputs (one 128-byte line) from registers.
//
// Measured on C4 (one B200, bit-exact against the streaming kernel): 179 us
// against 153-162 us (232 us before the epilogue read its row scales as
// shared-memory broadcasts, dropped per-element bounds checks and moved to
// packed FP32x2 arithmetic).  Each 128-token sub-tile costs about 5.4 us
// (48 pair MMAs of N = 128, about 115 ns each) whether A comes from tensor
// or shared memory, and the same with one accumulator buffer; N = 64 was
// slower still (296 us with four k-blocks per commit, 367 us with one).  Pair
// MMAs narrower than N = 256 do not reach the tensor peak, and N = 256 with
// two accumulator buffers fills the whole 512 TMEM columns.
//
// Work: the pair's 256-column weight tiles (NT of them) times the 128-token
// sub-tiles (MS) form S = NT x MS sub-tiles in (tile, token) order; pair p takes
// the contiguous range [p S / P, (p+1) S / P), so it loads a new weight tile at
// most a few times.  The epilogue warps load its TMEM part (plain loads ->
// tcgen05.st) and the producer its shared-memory part, after the MMAs reading
// the previous tile have completed.
#include "epilogue.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace htpg {

namespace {

constexpr int kTwEpiWarps = 16;
constexpr int kTwThreads = 64 + 32 * kTwEpiWarps;  // warp 0 TMA, warp 1 MMA, 2..17 epilogue
constexpr int kTwBM = 128;                         // tokens per sub-tile (MMA N)
constexpr int kTwRows = kTwBM / 2;                 // activation rows each CTA loads per k-block
// A stage holds up to kTwKbs k-blocks: each stage costs one MMA commit, and a
// commit costs about as much as a dozen small MMAs, so stages are large.
constexpr int kTwKbs = 4;
constexpr int kTwStages = 4;
constexpr uint32_t kTwKbBytes = kTwRows * 128;           // one k-block of this CTA's rows
constexpr uint32_t kTwStageBytes = kTwKbs * kTwKbBytes;  // per CTA
// The weight tile: its first kTwTmemKb k-blocks in TMEM columns [256, 512)
// (the two 128-column accumulators take [0, 256)), the rest (K > 1024, at
// most kTwSmemKb k-blocks) resident in shared memory, loaded once per tile.
constexpr int kTwTmemKb = 8;
constexpr int kTwSmemKb = 4;
constexpr uint32_t kTwACol = 256;
constexpr uint32_t kTwWKbBytes = 128 * 128;               // one k-block of this CTA's 128 weight rows
constexpr uint32_t kTwIdesc = idesc_i8(256, kTwBM);
// tail: barriers (first 512 bytes), then one 32-float row-scale slot per epilogue warp
constexpr size_t kTwSmem = 1024 + static_cast<size_t>(kTwStages) * kTwStageBytes +
                           static_cast<size_t>(kTwSmemKb) * kTwWKbBytes + 512 + kTwEpiWarps * 128;

struct TwParams {
  GemmArgs a;
  int MS;        // 64-token sub-tiles
  int NT;        // 256-column weight tiles
  long long S;   // NT * MS
  int KB;        // k-blocks (<= 12)
};

__device__ __forceinline__ void umma_i8_pair_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                    uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 lanes x 32 columns from registers: thread t writes lane (taddr.lane + t).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Packed FP32x2 arithmetic (two tokens of one output column per instruction).
// Each lane is the IEEE round-to-nearest operation of the scalar form, so
// finish2 gives the bits of finish (epilogue.cuh) for both elements.  The bias
// add stays scalar (__fadd_rn): a packed add after a packed multiply was
// measured to be contracted into one fused multiply-add (one rounding instead
// of two), which changes the bits.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float &a, float &b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// finish<Kind::I8, MODE, BIAS> for two accumulators of the same column.
template <int MODE, bool BIAS>
__device__ __forceinline__ void finish2(uint32_t a0, uint32_t a1, int32_t cr, uint64_t sw2, float rs0, float rs1,
                                        float bias, float &o0, float &o1) {
  const int32_t y0 = static_cast<int32_t>(a0 + static_cast<uint32_t>(cr));
  const int32_t y1 = static_cast<int32_t>(a1 + static_cast<uint32_t>(cr));
  if constexpr (MODE == 4) {
    o0 = __int_as_float(y0);
    o1 = __int_as_float(y1);
    return;
  } else {
    uint64_t v = mul2(mul2(pk2(__int2float_rn(y0), __int2float_rn(y1)), sw2), pk2(rs0, rs1));
    if constexpr (BIAS) {
      float v0, v1;
      upk2(v, v0, v1);
      v = pk2(__fadd_rn(v0, bias), __fadd_rn(v1, bias));
    }
    if constexpr (MODE == 1 || MODE == 2) {
      uint64_t h;
      if constexpr (MODE == 1) {
        constexpr float c1 = 0.5f * 1.5957691216057308f, c3 = 0.5f * 1.5957691216057308f * 0.044715f;
        h = mul2(v, fma2(mul2(v, v), pk2(c3, c3), pk2(c1, c1)));
      } else {
        h = mul2(v, pk2(0.5f * 1.702f, 0.5f * 1.702f));
      }
      float h0, h1;
      upk2(h, h0, h1);
      const uint64_t hx = mul2(pk2(0.5f, 0.5f), v);
      v = fma2(hx, pk2(tanh_approx(h0), tanh_approx(h1)), hx);
    }
    upk2(v, o0, o1);
  }
}

// One epilogue warp's 32 tokens x 32 columns of a finished sub-tile.  rs: the
// 32 row scales of those tokens in this warp's shared-memory slot (read as
// broadcast float4).  A full slice stores without per-element checks.
template <int MODE, bool BIAS>
__device__ __forceinline__ void tw_store(const GemmArgs &g, const uint32_t (&r)[32], int m0, int n, float sw,
                                         int32_t cr, float bv, const float *rs) {
  if (n >= g.N) return;
  float *p = g.out + static_cast<long long>(m0) * g.ldo + n;
  const long long ldo = g.ldo;
  if (m0 + 32 <= g.M) {
    const uint64_t sw2 = pk2(sw, sw);
#pragma unroll
    for (int j4 = 0; j4 < 8; ++j4) {
      const float4 s4 = *reinterpret_cast<const float4 *>(rs + 4 * j4);
      float o0, o1, o2, o3;
      finish2<MODE, BIAS>(r[4 * j4], r[4 * j4 + 1], cr, sw2, s4.x, s4.y, bv, o0, o1);
      finish2<MODE, BIAS>(r[4 * j4 + 2], r[4 * j4 + 3], cr, sw2, s4.z, s4.w, bv, o2, o3);
      p[0] = o0;
      p[ldo] = o1;
      p[2 * ldo] = o2;
      p[3 * ldo] = o3;
      p += 4 * ldo;
    }
  } else {
    for (int j = 0; j < 32 && m0 + j < g.M; ++j) {
      *p = finish<Kind::I8, MODE, BIAS>(r[j], cr, sw, rs[j], bv);
      p += ldo;
    }
  }
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTwThreads, 1)
    gemm_tw_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmW,
                   const TwParams P) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *wsm = ring + kTwStages * kTwStageBytes;  // resident weight k-blocks kTwTmemKb..
  uint64_t *bars = reinterpret_cast<uint64_t *>(wsm + kTwSmemKb * kTwWKbBytes);
  uint64_t *full = bars, *empty = bars + kTwStages, *tfull = bars + 2 * kTwStages,
           *tempty = bars + 2 * kTwStages + 2, *wready = bars + 2 * kTwStages + 4,
           *afree = bars + 2 * kTwStages + 5, *mma_done = bars + 2 * kTwStages + 6,
           *sready = bars + 2 * kTwStages + 7;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kTwStages + 8);
  float *rs_slots = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(bars) + 512);
  const int KT = min(P.KB, kTwTmemKb);  // weight k-blocks in TMEM; [KT, KB) in shared memory
  volatile uint32_t *abort = tmem_slot + 1;

  const GemmArgs &g = P.a;
  uint32_t *wd = g.watchdog;
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const long long s0 = P.S * pair / npairs, s1 = P.S * (pair + 1) / npairs;
  const uint32_t peer_abort = mapa_shared(smem_u32(const_cast<uint32_t *>(abort)), rank ^ 1u);
  grid_dependents_launch();
  auto wait = [&](uint32_t bar, uint32_t parity, uint32_t bit) {
    const bool ok = mbar_wait(bar, parity, wd, bit, abort);
    if (!ok) st_shared_cluster(peer_abort, 1u);
    return ok;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTwStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), 2 * kTwEpiWarps);
    }
    mbar_init(smem_u32(wready), 2 * kTwEpiWarps);
    mbar_init(smem_u32(afree), 1);
    mbar_init(smem_u32(mma_done), 1);
    mbar_init(smem_u32(sready), 1);
    *abort = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tmB);
      tma_prefetch_desc(&tmW);
      grid_dependency_wait();  // the codes come from the activation pass
      int s = 0;
      uint32_t ph = 0, loads = 0;
      long long cur_nt = -1;
      int last_phase[kTwStages];
      for (int i = 0; i < kTwStages; ++i) last_phase[i] = -1;
      bool ok = true;
      bool w_pending = false;  // a resident-weight load may still be landing
      for (long long st = s0; ok && st < s1; ++st) {
        const long long nt = st / P.MS;
        if (nt != cur_nt && P.KB > KT) {
          // the k-blocks past KT of this CTA's 128 weight rows, once per tile,
          // after the MMAs that read the previous tile's have completed
          if (loads > 0 && !wait(smem_u32(afree), (loads - 1) & 1u, kWatchProducer)) break;
          const uint32_t sb = smem_u32(sready);
          if (leader) mbar_arrive_expect_tx(sb, 2u * (P.KB - KT) * kTwWKbBytes);
          for (int kb = KT; kb < P.KB; ++kb)
            tma_load_2d_pair(smem_u32(wsm + (kb - KT) * kTwWKbBytes), &tmW, mapa_shared(sb, 0), 0,
                             kb * g.N + static_cast<int>(nt) * 256 + static_cast<int>(rank) * 128);
          w_pending = true;
          ++loads;
        }
        cur_nt = nt;
        const int m0 = static_cast<int>(st % P.MS) * kTwBM;
        for (int kb0 = 0; kb0 < P.KB; kb0 += kTwKbs) {
          if (!wait(smem_u32(&empty[s]), ph ^ 1u, kWatchProducer)) {
            ok = false;
            break;
          }
          const int nk = min(kTwKbs, P.KB - kb0);
          const uint32_t fb_local = smem_u32(&full[s]);
          if (leader) mbar_arrive_expect_tx(fb_local, 2u * nk * kTwKbBytes);
          for (int j = 0; j < nk; ++j)
            tma_load_2d_pair(smem_u32(ring + s * kTwStageBytes + j * kTwKbBytes), &tmB, mapa_shared(fb_local, 0),
                             (kb0 + j) * 128, m0 + static_cast<int>(rank) * kTwRows);
          last_phase[s] = static_cast<int>(ph);
          if (++s == kTwStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // the leader's full barriers count both CTAs' bytes: once they complete,
      // no copy is still landing in either CTA
      if (leader) {
        for (int i = 0; i < kTwStages; ++i)
          if (last_phase[i] >= 0) wait(smem_u32(&full[i]), static_cast<uint32_t>(last_phase[i]), kWatchProducer);
        if (w_pending) wait(smem_u32(sready), (loads - 1) & 1u, kWatchProducer);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (lane == 0 && leader) {
      grid_dependency_wait();
      int s = 0;
      uint32_t ph = 0, iter = 0, loads = 0;
      long long cur_nt = -1;
      bool ok = true;
      for (long long st = s0; ok && st < s1; ++st, ++iter) {
        const long long nt = st / P.MS;
        if (nt != cur_nt) {
          // the MMAs that read the previous weight tile have completed before
          // the epilogue warps overwrite it; then wait for the new one
          if (loads > 0) tc_commit_pair_mc(smem_u32(afree), 0x3);
          if (!wait(smem_u32(wready), loads & 1u, kWatchMma)) break;
          if (P.KB > KT && !wait(smem_u32(sready), loads & 1u, kWatchMma)) break;
          tc_fence_after();
          cur_nt = nt;
          ++loads;
        }
        const uint32_t buf = iter & 1u;
        if (!wait(smem_u32(&tempty[buf]), ((iter >> 1) & 1u) ^ 1u, kWatchMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kTwBM;
        for (int kb0 = 0; kb0 < P.KB; kb0 += kTwKbs) {
          if (!wait(smem_u32(&full[s]), ph, kWatchMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nk = min(kTwKbs, P.KB - kb0);
          for (int j = 0; j < nk; ++j) {
            const int kb = kb0 + j;
            const uint32_t b_addr = smem_u32(ring + s * kTwStageBytes + j * kTwKbBytes);
            if (kb < KT) {
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_i8_pair_tmem_a(d_tmem, tmem_base + kTwACol + kb * 32 + kk * 8,
                                    umma_desc_sw128(b_addr + kk * 32), kTwIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
            } else {
              const uint32_t a_addr = smem_u32(wsm + (kb - KT) * kTwWKbBytes);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk)
                umma_i8_pair(d_tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32), kTwIdesc,
                             1u);
            }
          }
          tc_commit_pair_mc(smem_u32(&empty[s]), 0x3);
          if (++s == kTwStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (ok) tc_commit_pair_mc(smem_u32(&tfull[buf]), 0x3);
      }
      tc_commit_pair(smem_u32(mma_done));
      wait(smem_u32(mma_done), 0, kWatchMma);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;          // TMEM lane quadrant
    const int part = (warp - 2) / 4;  // 32-token slice of the sub-tile; k-blocks part, part + 4, ...
    const uint32_t lane_addr = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t wready_leader = mapa_shared(smem_u32(wready), 0);
    const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&tempty[0]), 0), mapa_shared(smem_u32(&tempty[1]), 0)};
    const int8_t *wk = static_cast<const int8_t *>(g.wk);
    const int mode = g.mode;
    const bool has_bias = g.bias != nullptr;
    long long cur_nt = -1;
    uint32_t loads = 0, iter = 0;
    int n = 0;
    float sw = 0.f, bv = 0.f;
    int32_t cr = 0;
    bool waited = false;
    for (long long st = s0; st < s1; ++st, ++iter) {
      const long long nt = st / P.MS;
      if (nt != cur_nt) {
        if (loads > 0 && !mbar_wait(smem_u32(afree), (loads - 1) & 1u, wd, kWatchEpilogue, abort)) {
          st_shared_cluster(peer_abort, 1u);
          break;
        }
        tc_fence_after();
        // this CTA's 128 columns of the tile: lane = column, 32 TMEM columns
        // (128 bytes of K) per k-block; the weights do not depend on the
        // previous kernel, so the first tile loads before its dependency wait
        n = static_cast<int>(nt) * 256 + static_cast<int>(rank) * 128 + q * 32 + lane;
        for (int kb = part; kb < KT; kb += 4) {
          uint32_t w[32];
          if (n < g.N) {
            const uint4 *src = reinterpret_cast<const uint4 *>(wk + (static_cast<size_t>(kb) * g.N + n) * 128u);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint4 v = __ldg(src + i);
              w[4 * i] = v.x;
              w[4 * i + 1] = v.y;
              w[4 * i + 2] = v.z;
              w[4 * i + 3] = v.w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = 0u;
          }
          tmem_st32(tmem_base + lane_addr + kTwACol + static_cast<uint32_t>(kb) * 32u, w);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(wready_leader);
        if (!waited) {
          grid_dependency_wait();  // row scales come from the activation pass
          waited = true;
        }
        sw = n < g.N ? __ldg(g.col_scale + n) : 0.f;
        cr = n < g.N ? __ldg(g.col_corr + n) : 0;
        bv = (has_bias && n < g.N) ? __ldg(g.bias + n) : 0.f;
        cur_nt = nt;
        ++loads;
      }
      const int m0 = static_cast<int>(st % P.MS) * kTwBM + part * 32;
      float *rs_slot = rs_slots + (warp - 2) * 32;
      __syncwarp();  // the previous sub-tile's reads of the slot are done
      rs_slot[lane] = m0 + lane < g.M ? __ldg(g.row_scale + m0 + lane) : 0.f;
      __syncwarp();
      const uint32_t buf = iter & 1u;
      if (!mbar_wait(smem_u32(&tfull[buf]), (iter >> 1) & 1u, wd, kWatchEpilogue, abort)) {
        st_shared_cluster(peer_abort, 1u);
        break;
      }
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tmem_base + lane_addr + buf * kTwBM + part * 32, r);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[buf]);
      switch (mode * 2 + (has_bias ? 1 : 0)) {
        case 0: tw_store<0, false>(g, r, m0, n, sw, cr, bv, rs_slot); break;
        case 1: tw_store<0, true>(g, r, m0, n, sw, cr, bv, rs_slot); break;
        case 2: tw_store<1, false>(g, r, m0, n, sw, cr, bv, rs_slot); break;
        case 3: tw_store<1, true>(g, r, m0, n, sw, cr, bv, rs_slot); break;
        case 4: tw_store<2, false>(g, r, m0, n, sw, cr, bv, rs_slot); break;
        case 5: tw_store<2, true>(g, r, m0, n, sw, cr, bv, rs_slot); break;
        default: tw_store<4, false>(g, r, m0, n, sw, cr, bv, rs_slot); break;
      }
    }
  }

  // every MMA (which read both CTAs' shared and tensor memory) and every TMEM
  // access is complete before either CTA releases TMEM or exits
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
}

}  // namespace

bool tw_eligible(const GemmPlan &p, int mode, int n_outs) {
  return p.kind == Kind::I8 && p.pair && p.kb_total <= 12 && n_outs == 1 &&
         (mode == 0 || mode == 1 || mode == 2 || mode == 4);
}

int tw_box_rows() { return kTwRows; }

cudaError_t launch_gemm_tw(const GemmPlan &p, const CUtensorMap &tmB, const CUtensorMap &tmW, const GemmArgs &a,
                           cudaStream_t st) {
  static bool configured[64] = {};
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm_tw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kTwSmem));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  TwParams P;
  P.a = a;
  P.MS = (a.M + kTwBM - 1) / kTwBM;
  P.NT = (a.N + 255) / 256;
  P.S = static_cast<long long>(P.MS) * P.NT;
  P.KB = p.kb_total;
  const int pairs = sms[dev] / 2;  // one CTA pair per two SMs, over 64-token sub-tiles
  const long long grid = 2 * (P.S < pairs ? P.S : pairs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kTwThreads, 1, 1);
  cfg.dynamicSmemBytes = kTwSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tw_kernel, tmB, tmW, P);
  return counted(e != cudaSuccess ? e : cudaGetLastError());
}

}  // namespace htpg
