// Opcode 19: FP32 model auxiliaries around the linears (reference:
// src/dsp/ops/mat_mul.c:2344-2480 model_aux_worker, validation
// src/dsp/op_executor.cc:371-395).  Memory-bound elementwise and row-reduction
// kernels; the norms reduce with FP32 partial sums per thread and FP64 block
// sums, as the reference sums its FP32 lanes in double.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/htp_ops_b200.h"
#include "../../include/op_reg.h"

namespace {

struct AuxArgs {
  int mode, count, width, channels, spatial, groups, batch, other, act;
  float eps;
};

// x*sigmoid(z) with the reference's stable split (mat_mul.c:788-826):
// e = 2^(-|z| log2 e) clamped at 2^-126, sigmoid = z < 0 ? e/(1+e) : 1/(1+e).
// mode 1 GELU(tanh), 2 QuickGELU, 4/5 SiLU.
__device__ __forceinline__ float act_fn(float x, int mode) {
  float z = x;
  if (mode == 1) z = x + (x * x * x) * 0.044715f;
  z = z * (mode == 1 ? 1.5957691216057308f : (mode == 4 || mode == 5) ? 1.0f : 1.702f);
  const float neg = fmaxf(fabsf(z) * -1.4426950408889634f, -126.0f);
  const float e = exp2f(neg);
  const float inv = 1.0f / (e + 1.0f);
  return x * (z < 0.0f ? e * inv : inv);
}

constexpr int kNormThreads = 256;

__device__ double block_sum(double v, double *red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by the previous reduction
  if (lane == 0) red[w] = v;
  __syncthreads();
  double s = 0.0;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) s += red[i];
  return s;
}

// Modes 0 (LayerNorm), 1 (RMSNorm), 2 (GroupNorm), 9 (LayerNorm + modulation):
// one block per row (modes 0, 1, 9) or per (batch, group) (mode 2).
__global__ void __launch_bounds__(kNormThreads) aux_norm_kernel(float *__restrict__ out,
                                                                const float *__restrict__ x,
                                                                const float *__restrict__ w,
                                                                const float *__restrict__ b, AuxArgs a) {
  __shared__ double red[kNormThreads / 32];
  const long long n = a.mode == 2 ? static_cast<long long>(a.spatial) * (a.channels / a.groups) : a.width;
  const long long task = blockIdx.x;
  const long long off = task * n;
  const float *xr = x + off;
  float mean = 0.0f;
  if (a.mode != 1) {
    float s = 0.0f;
    for (long long i = threadIdx.x; i < n; i += kNormThreads) s += xr[i];
    mean = static_cast<float>(block_sum(s, red) / static_cast<double>(n));
  }
  float q = 0.0f;
  for (long long i = threadIdx.x; i < n; i += kNormThreads) {
    const float d = xr[i] - mean;
    q += d * d;
  }
  const float inv = 1.0f / sqrtf(static_cast<float>(block_sum(q, red) / static_cast<double>(n) + a.eps));
  const long long pb = (a.mode == 9 && a.other != a.width) ? task / a.spatial : 0;
  for (long long i = threadIdx.x; i < n; i += kNormThreads) {
    float v = (xr[i] - mean) * inv;
    if (a.mode == 2) {
      const int ch = static_cast<int>(((off + i) / a.spatial) % a.channels);
      if (w) v = v * w[ch];
      if (b) v = v + b[ch];
    } else if (a.mode == 9) {
      v = v + v * w[pb * a.width + i];
      v = v + b[pb * a.width + i];
    } else {
      if (w) v = v * w[i];
      if (b) v = v + b[i];
    }
    if (a.act) v = act_fn(v, 4);
    out[off + i] = v;
  }
}

// Rows of at most 16*256 floats (modes 0, 1, 9): the row is read once into
// registers, then reduced and normalised from there.
template <int PER>
__global__ void __launch_bounds__(kNormThreads) aux_row_norm_reg_kernel(float *__restrict__ out,
                                                                       const float *__restrict__ x,
                                                                       const float *__restrict__ w,
                                                                       const float *__restrict__ b, AuxArgs a) {
  __shared__ double red[kNormThreads / 32];
  const int n = a.width;
  const long long task = blockIdx.x;
  const float *xr = x + task * n;
  float v[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = j * kNormThreads + threadIdx.x;
    v[j] = i < n ? xr[i] : 0.0f;
  }
  float mean = 0.0f;
  if (a.mode != 1) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < PER; ++j) s += v[j];
    mean = static_cast<float>(block_sum(s, red) / static_cast<double>(n));
  }
  float q = 0.0f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = j * kNormThreads + threadIdx.x;
    const float d = i < n ? v[j] - mean : 0.0f;
    q += d * d;
  }
  const float inv = 1.0f / sqrtf(static_cast<float>(block_sum(q, red) / static_cast<double>(n) + a.eps));
  const long long pb = (a.mode == 9 && a.other != a.width) ? task / a.spatial : 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int i = j * kNormThreads + threadIdx.x;
    if (i >= n) break;
    float y = (v[j] - mean) * inv;
    if (a.mode == 9) {
      y = y + y * w[pb * a.width + i];
      y = y + b[pb * a.width + i];
    } else {
      if (w) y = y * w[i];
      if (b) y = y + b[i];
    }
    if (a.act) y = act_fn(y, 4);
    out[task * n + i] = y;
  }
}

// Mode 12 (SwiGLU) with rows and 4-column groups: grid.y = row.
__global__ void aux_swiglu_kernel(float *__restrict__ out, const float *__restrict__ x, AuxArgs a) {
  const long long row = blockIdx.y;
  const int c4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (c4 >= a.width) return;
  const float *r = x + row * a.channels + c4;
  const float4 p = *reinterpret_cast<const float4 *>(r);
  const float4 q = *reinterpret_cast<const float4 *>(r + a.width);
  const float4 gate = a.act ? p : q, up = a.act ? q : p;
  *reinterpret_cast<float4 *>(out + row * a.width + c4) =
      make_float4(act_fn(gate.x, 5) * up.x, act_fn(gate.y, 5) * up.y, act_fn(gate.z, 5) * up.z,
                  act_fn(gate.w, 5) * up.w);
}

// Elementwise modes: 3/4 broadcast add/multiply, 5/6/7 activations, 10 gated
// residual, 12 SwiGLU, 13 attention copy + SwiGLU.
__global__ void aux_elementwise_kernel(float *__restrict__ out, const float *__restrict__ x,
                                       const float *__restrict__ w, const float *__restrict__ b, AuxArgs a) {
  const long long total = a.count;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float v;
    switch (a.mode) {
      case 3: v = x[i] + w[i % a.other]; break;
      case 4: v = x[i] * w[i % a.other]; break;
      case 5: v = act_fn(x[i], 4); break;
      case 6: v = act_fn(x[i], 1); break;
      case 7: v = act_fn(x[i], 2); break;
      case 10: {
        const int ch = static_cast<int>(i % a.width);
        const long long pb = a.other == a.width ? 0 : i / (static_cast<long long>(a.width) * a.spatial);
        v = x[i] * w[pb * a.width + ch] + b[i];
        break;
      }
      case 12: {
        const long long row = i / a.width, col = i % a.width;
        const float *r = x + row * a.channels + col;
        const float gate = a.act ? r[0] : r[a.width], up = a.act ? r[a.width] : r[0];
        v = act_fn(gate, 5) * up;
        break;
      }
      default: {  // 13
        const int ow = a.width + a.groups;
        const long long row = i / ow, col = i % ow;
        if (col < a.groups) {
          v = w[row * a.groups + col];
        } else {
          const float *r = x + row * a.channels + (col - a.groups);
          const float gate = a.act ? r[0] : r[a.width], up = a.act ? r[a.width] : r[0];
          v = act_fn(gate, 5) * up;
        }
      }
    }
    out[i] = v;
  }
}

// Mode 8: [batch][width][spatial] -> [batch][spatial][width], 32 x 32 tiles.
__global__ void aux_transpose_kernel(float *__restrict__ out, const float *__restrict__ x, AuxArgs a) {
  __shared__ float tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32, bb = blockIdx.z;
  const float *xb = x + static_cast<long long>(bb) * a.width * a.spatial;
  float *ob = out + static_cast<long long>(bb) * a.width * a.spatial;
  for (int rr = threadIdx.y; rr < 32; rr += 8) {
    const int r = r0 + rr, c = c0 + threadIdx.x;
    if (r < a.width && c < a.spatial) tile[rr][threadIdx.x] = xb[static_cast<long long>(r) * a.spatial + c];
  }
  __syncthreads();
  for (int cc = threadIdx.y; cc < 32; cc += 8) {
    const int c = c0 + cc, r = r0 + threadIdx.x;
    if (r < a.width && c < a.spatial) ob[static_cast<long long>(c) * a.width + r] = tile[threadIdx.x][cc];
  }
}

// Mode 11: rotary position embedding with a 2x2 matrix per element pair,
// input [batch][token][head][dim] -> output [batch][head][token][dim].
__global__ void aux_rope_kernel(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ pe,
                                AuxArgs a) {
  const int dim = a.width, heads = a.channels, pairs = dim / 2;
  const long long total = static_cast<long long>(a.batch) * a.spatial * heads * pairs;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int e = static_cast<int>(i % pairs) * 2;
    long long rest = i / pairs;
    const int h = static_cast<int>(rest % heads);
    rest /= heads;
    const int tok = static_cast<int>(rest % a.spatial);
    const int bb = static_cast<int>(rest / a.spatial);
    const float *m = pe + (static_cast<long long>(a.groups == 1 ? 0 : bb) * a.spatial + tok) * dim * 2 + 2 * e;
    const float *xi = x + ((static_cast<long long>(bb) * a.spatial + tok) * heads + h) * dim;
    float *o = out + ((static_cast<long long>(bb) * heads + h) * a.spatial + tok) * dim;
    const float x0 = xi[e], x1 = xi[e + 1];
    o[e] = x0 * m[0] + x1 * m[1];
    o[e + 1] = x1 * m[3] + x0 * m[2];
  }
}

}  // namespace

// Geometry and operand checks of the reference executor (op_executor.cc:375-395);
// w/b presence stands for weight.fd/bias.fd >= 0.
extern "C" int htpg_model_aux_check(const struct NativeAuxParams *p, int has_w, int has_b) {
  if (!p) return HTPG_EARGS;
  if (p->count <= 0 || p->mode < 0 || p->mode > 13 || p->width <= 0 || p->channels <= 0 || p->spatial <= 0 ||
      p->batch <= 0)
    return HTPG_EPAYLOAD;
  const int64_t wsb = static_cast<int64_t>(p->width) * p->spatial * p->batch;
  if (p->mode == 8 && wsb != p->count) return HTPG_EPAYLOAD;
  if (p->mode == 2 && (p->groups <= 0 || p->channels % p->groups)) return HTPG_EPAYLOAD;
  if (p->mode == 12 && (wsb != p->count || has_w || has_b || p->channels < 2LL * p->width ||
                        (p->activation != 0 && p->activation != 1)))
    return HTPG_EPAYLOAD;
  if (p->mode == 13 && (p->groups <= 0 || !has_w || has_b ||
                        (static_cast<int64_t>(p->width) + p->groups) * p->spatial * p->batch != p->count ||
                        static_cast<int64_t>(p->groups) * p->spatial * p->batch != p->other_count ||
                        p->channels < 2LL * p->width || (p->activation != 0 && p->activation != 1)))
    return HTPG_EPAYLOAD;
  if ((p->mode == 9 || p->mode == 10) &&
      (wsb != p->count || !has_w || !has_b ||
       (p->other_count != p->width && p->other_count != static_cast<int64_t>(p->width) * p->batch) ||
       (p->mode == 9 && (!std::isfinite(p->eps) || p->eps < 0))))
    return HTPG_EPAYLOAD;
  if (p->mode == 11 && (p->width % 2 || static_cast<int64_t>(p->width) * p->channels * p->spatial * p->batch != p->count ||
                        !has_w || has_b || (p->groups != 1 && p->groups != p->batch) ||
                        p->other_count != 2LL * p->width * p->spatial * p->groups))
    return HTPG_EPAYLOAD;
  const int n = p->mode == 2 ? p->channels : p->mode == 9 ? p->other_count : p->mode == 10 ? p->count : p->width;
  if (p->mode <= 2 && has_w && p->other_count != n) return HTPG_EPAYLOAD;
  if ((p->mode == 3 || p->mode == 4) && (p->other_count <= 0 || p->count % p->other_count || !has_w))
    return HTPG_EPAYLOAD;
  // GroupNorm reads spatial*channels*batch elements: stricter than the
  // reference, which would read and write past a shorter tensor
  if (p->mode == 2 && static_cast<int64_t>(p->spatial) * p->channels * p->batch != p->count) return HTPG_EPAYLOAD;
  return HTPG_OK;
}

extern "C" int htpg_model_aux(float *dst, const float *x, const float *w, const float *b,
                              const struct NativeAuxParams *p, void *stream) {
  if (!dst || !x || !p) return HTPG_EARGS;
  int rc = htpg_model_aux_check(p, w != nullptr, b != nullptr);
  if (rc) return rc;
  const AuxArgs a = {p->mode,    p->count, p->width,       p->channels,   p->spatial,
                     p->groups, p->batch, p->other_count, p->activation, p->eps};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((a.mode <= 1 || a.mode == 9) && a.width <= 16 * kNormThreads) {
    const unsigned tasks = static_cast<unsigned>(a.count / a.width);
    const int per = (a.width + kNormThreads - 1) / kNormThreads;
    if (per <= 2)
      aux_row_norm_reg_kernel<2><<<tasks, kNormThreads, 0, st>>>(dst, x, w, b, a);
    else if (per <= 4)
      aux_row_norm_reg_kernel<4><<<tasks, kNormThreads, 0, st>>>(dst, x, w, b, a);
    else if (per <= 8)
      aux_row_norm_reg_kernel<8><<<tasks, kNormThreads, 0, st>>>(dst, x, w, b, a);
    else
      aux_row_norm_reg_kernel<16><<<tasks, kNormThreads, 0, st>>>(dst, x, w, b, a);
  } else if (a.mode <= 2 || a.mode == 9) {
    const long long tasks = a.mode == 2 ? static_cast<long long>(a.groups) * a.batch : a.count / a.width;
    aux_norm_kernel<<<static_cast<unsigned>(tasks), kNormThreads, 0, st>>>(dst, x, w, b, a);
  } else if (a.mode == 12 && a.width % 4 == 0 && a.channels % 4 == 0 &&
             (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
    const long long rows = a.count / a.width;
    const dim3 grid(static_cast<unsigned>((a.width / 4 + 255) / 256), static_cast<unsigned>(rows));
    aux_swiglu_kernel<<<grid, 256, 0, st>>>(dst, x, a);
  } else if (a.mode == 8) {
    const dim3 grid((a.spatial + 31) / 32, (a.width + 31) / 32, a.batch);
    aux_transpose_kernel<<<grid, dim3(32, 8), 0, st>>>(dst, x, a);
  } else if (a.mode == 11) {
    const long long total = static_cast<long long>(a.batch) * a.spatial * a.channels * (a.width / 2);
    aux_rope_kernel<<<static_cast<unsigned>((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096), 256, 0, st>>>(
        dst, x, w, a);
  } else {
    const long long total = a.count;
    aux_elementwise_kernel<<<static_cast<unsigned>((total + 255) / 256 < 8192 ? (total + 255) / 256 : 8192), 256, 0,
                             st>>>(dst, x, w, b, a);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? HTPG_OK : HTPG_ELAUNCH;
}

extern "C" int hvx_model_aux_f32(float *dst, const float *x, const float *w, const float *b,
                                 const struct NativeAuxParams *p) {
  const int rc = htpg_model_aux(dst, x, w, b, p, nullptr);
  if (rc) return rc;
  return cudaStreamSynchronize(nullptr) == cudaSuccess ? HTPG_OK : HTPG_ELAUNCH;
}
