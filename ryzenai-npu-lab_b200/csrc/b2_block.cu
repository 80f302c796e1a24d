// B200 (sm_100a) kernels of the LFM2.5 layer around the attention hot path:
//
//   add_rmsnorm_kernel    residual add + RMSNorm (one CTA of 128 threads per row)
//   swiglu_kernel         silu(w1 x) * (w3 x), 8 values per thread
//   shortconv_step_kernel one decode step of the gated short convolution
//   argmax_rows_kernel    greedy token choice over the vocabulary logits
//
// Each replaces a chain of small framework kernels between the layer's
// GEMMs; the rounding points are those of the bf16 tensors of the model
// definition (transformers modeling_lfm2.py, see include/b2_block.h).

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "b2_block.h"
#include "b2_decode_attn.h"
#include "b2_internal.h"

namespace {

constexpr int kNormThreads = 128;
constexpr int kNormMaxChunks = 4;  // 8-value chunks per thread: width <= 128 * 8 * 4

__device__ __forceinline__ float bf2f(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// Let a kernel launched after this one with programmatic stream serialization
// (b2_gemm) start its own set-up and its weight copies now; it reads this
// kernel's output only after griddepcontrol.wait, which waits for this grid
// to complete.
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t f2bf(float x) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x)));
}

__device__ __forceinline__ float rnd(float x) { return bf2f(f2bf(x)); }

__device__ __forceinline__ void unpack8(const uint4 &w, float f[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float f[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t *>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Sum of the squares of one row, bit-identical to torch's CPU
// x.pow(2).mean(-1) * width for a contiguous row of `width` floats (a multiple
// of 32, at most 4096): ATen's vectorised inner sum over 8-float vectors v_m
// (elements 8m..8m+7), read as rows of 4 vectors (row i = v_4i..v_4i+3)
// summed into 4 lane-wise accumulators in a cascade of 16-row groups:
//   S_gk = v_{4(16g)+k} + ... + v_{4(16g+15)+k}   (left to right from 0)
//   A_k  = S_0k + S_1k + ...                      (left to right)
//   P_k  = (rows past the last full group, left to right from 0) + A_k
//   p    = ((P_0 + P_1) + P_2) + P_3, then its 8 lanes left to right.
// sq holds the row's rounded squares; every thread of the CTA calls this.
__device__ float torch_order_sum(const float *sq, int width, float *chains) {
  const int rows = width / 32;
  const int groups = rows / 16, tail = rows % 16;
  const int nchains = (groups + (tail > 0)) * 32;  // (group, k, lane)
  for (int c = threadIdx.x; c < nchains; c += blockDim.x) {
    const int g = c >> 5, k = (c >> 3) & 3, l = c & 7;
    const int r0 = 16 * g, r1 = g < groups ? r0 + 16 : r0 + tail;
    float acc = sq[(4 * r0 + k) * 8 + l];
    for (int i = r0 + 1; i < r1; ++i) acc = __fadd_rn(acc, sq[(4 * i + k) * 8 + l]);
    chains[c] = acc;
  }
  __syncthreads();
  float total = 0.f;
  if (threadIdx.x < 32) {
    const int k = threadIdx.x >> 3, l = threadIdx.x & 7;
    float a = chains[threadIdx.x];
    for (int g = 1; g < groups; ++g) a = __fadd_rn(a, chains[g * 32 + threadIdx.x]);
    const float P = tail > 0 ? (groups > 0 ? __fadd_rn(chains[groups * 32 + threadIdx.x], a)
                                           : chains[threadIdx.x])
                             : a;
    // p_l = ((P_0l + P_1l) + P_2l) + P_3l on lanes l = 0..7 (lane 8k + l holds P_kl)
    const float p1 = __shfl_sync(0xffffffffu, P, 8 + l);
    const float p2 = __shfl_sync(0xffffffffu, P, 16 + l);
    const float p3 = __shfl_sync(0xffffffffu, P, 24 + l);
    const float pl = __fadd_rn(__fadd_rn(__fadd_rn(P, p1), p2), p3);
    total = __shfl_sync(0xffffffffu, pl, 0);
#pragma unroll
    for (int j = 1; j < 8; ++j) total = __fadd_rn(total, __shfl_sync(0xffffffffu, pl, j));
    (void)k;
    if (threadIdx.x == 0) chains[0] = total;
  }
  __syncthreads();
  return chains[0];
}

// sum_out may alias x or residual: every thread reads its own chunks before
// the barrier and writes only those chunks after it.
// Lfm2RMSNorm: gamma * bf16(x * rsqrt(mean(x^2) + eps)) with the mean summed
// in torch's CPU order (widths that are a multiple of 32) and rsqrt as
// 1 / sqrt with IEEE-rounded sqrt and divide, as torch's CPU rsqrt computes it.
__global__ void __launch_bounds__(kNormThreads)
    add_rmsnorm_kernel(const uint16_t *x, const uint16_t *residual, const uint16_t *__restrict__ gamma,
                       float eps, uint16_t *sum_out, uint16_t *__restrict__ norm_out, int width) {
  __shared__ float sq[kNormThreads * 8 * kNormMaxChunks];
  __shared__ float chains[kNormThreads * 8 * kNormMaxChunks / 32 / 16 * 32 + 32];
  __shared__ float red[kNormThreads / 32];
  allow_dependents();
  const int64_t row = blockIdx.x;
  const int chunks = width / 8;
  const bool torch_order = width % 32 == 0;
  float v[kNormMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormMaxChunks; ++k) {
    const int c = threadIdx.x + k * kNormThreads;
    if (c < chunks) {
      unpack8(reinterpret_cast<const uint4 *>(x + row * width)[c], v[k]);
      if (residual) {
        float r[8];
        unpack8(reinterpret_cast<const uint4 *>(residual + row * width)[c], r);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k][e] = rnd(v[k][e] + r[e]);  // bf16 tensor add
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float q = __fmul_rn(v[k][e], v[k][e]);
        if (torch_order) sq[c * 8 + e] = q;
        else ss += q;
      }
    }
  }
  float tot;
  if (torch_order) {
    __syncthreads();
    tot = torch_order_sum(sq, width, chains);
  } else {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    tot = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) tot += red[w];
  }
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(width)), eps)));
#pragma unroll
  for (int k = 0; k < kNormMaxChunks; ++k) {
    const int c = threadIdx.x + k * kNormThreads;
    if (c < chunks) {
      if (sum_out) reinterpret_cast<uint4 *>(sum_out + row * width)[c] = pack8(v[k]);
      float g[8], o[8];
      unpack8(reinterpret_cast<const uint4 *>(gamma)[c], g);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(g[e], rnd(__fmul_rn(v[k][e], inv)));
      reinterpret_cast<uint4 *>(norm_out + row * width)[c] = pack8(o);
    }
  }
}

// silu(g) = g / (1 + e^-g) in fp32, rounded to bf16 as the bf16 silu tensor is
__global__ void swiglu_kernel(const uint16_t *__restrict__ gu, uint16_t *__restrict__ out, int rows, int ffn) {
  allow_dependents();
  const int chunks = ffn / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(rows) * chunks) return;
  const int64_t r = i / chunks;
  const int c = static_cast<int>(i - r * chunks);
  float g[8], u[8], o[8];
  unpack8(reinterpret_cast<const uint4 *>(gu + r * 2 * ffn)[c], g);
  unpack8(reinterpret_cast<const uint4 *>(gu + r * 2 * ffn + ffn)[c], u);
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(rnd(__fdiv_rn(g[e], 1.0f + expf(-g[e]))), u[e]);
  reinterpret_cast<uint4 *>(out + r * ffn)[c] = pack8(o);
}

// one thread per (row, channel); state [rows][hidden][3], weights [hidden][3]
__global__ void shortconv_step_kernel(const uint16_t *__restrict__ bcx, uint16_t *__restrict__ state,
                                      const uint16_t *__restrict__ w, uint16_t *__restrict__ out, int rows,
                                      int hidden) {
  allow_dependents();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t r = blockIdx.y;
  if (c >= hidden) return;
  const uint16_t *in = bcx + r * 3 * hidden;
  const float B = bf2f(in[c]), C = bf2f(in[hidden + c]), xx = bf2f(in[2 * hidden + c]);
  const float bx = rnd(B * xx);
  uint16_t *st = state + (r * hidden + c) * 3;
  const float s1 = bf2f(st[1]), s2 = bf2f(st[2]);
  st[0] = static_cast<uint16_t>(f2bf(s1));
  st[1] = static_cast<uint16_t>(f2bf(s2));
  st[2] = static_cast<uint16_t>(f2bf(bx));
  const float p0 = rnd(s1 * bf2f(w[c * 3])), p1 = rnd(s2 * bf2f(w[c * 3 + 1])), p2 = rnd(bx * bf2f(w[c * 3 + 2]));
  const float conv = rnd((p0 + p1) + p2);
  out[r * hidden + c] = static_cast<uint16_t>(f2bf(C * conv));
}

// (value, index) pairs: a beats b when larger, NaN beating numbers, and the
// smaller index on ties (torch.argmax's first maximum)
__device__ __forceinline__ bool better(float va, int ia, float vb, int ib) {
  const bool na = va != va, nb = vb != vb;
  if (na != nb) return na;
  if (!na && va != vb) return va > vb;
  return ia < ib;
}

constexpr int kArgmaxThreads = 512;

// one CTA per row; 8 values per 16-byte load (cols % 8 == 0)
__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_rows_kernel(const uint16_t *__restrict__ logits, int cols, int64_t *__restrict__ out) {
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
  allow_dependents();
  const int64_t row = blockIdx.x;
  const uint4 *p = reinterpret_cast<const uint4 *>(logits + row * cols);
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = threadIdx.x; c < cols / 8; c += kArgmaxThreads) {
    float v[8];
    unpack8(p[c], v);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (better(v[e], c * 8 + e, bv, bi)) {
        bv = v[e];
        bi = c * 8 + e;
      }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kArgmaxThreads / 32; ++w)
      if (better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
    out[row] = bi;
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launched(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return b2_record_error(B2_ERR_CUDA, what);
  return b2_clear_error();
}

}  // namespace

extern "C" int b2_add_rmsnorm(const uint16_t *x, const uint16_t *residual, const uint16_t *gamma, float eps,
                              uint16_t *sum_out, uint16_t *norm_out, int32_t rows, int32_t width, void *stream) {
  if (rows < 0) return b2_record_error(B2_ERR_ARG, "b2_add_rmsnorm: rows must be >= 0");
  if (rows == 0) return b2_clear_error();
  if (!x || !gamma || !norm_out) return b2_record_error(B2_ERR_ARG, "b2_add_rmsnorm: null pointer argument");
  if (width <= 0 || width % 8 || width > kNormThreads * 8 * kNormMaxChunks)
    return b2_record_error(B2_ERR_ARG, "b2_add_rmsnorm: width must be a positive multiple of 8, at most 4096");
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(norm_out) || (residual && !aligned16(residual)) ||
      (sum_out && !aligned16(sum_out)))
    return b2_record_error(B2_ERR_ARG, "b2_add_rmsnorm: pointers must be 16-byte aligned");
  if (!(eps >= 0.f)) return b2_record_error(B2_ERR_ARG, "b2_add_rmsnorm: eps must be >= 0");
  add_rmsnorm_kernel<<<rows, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(x, residual, gamma, eps, sum_out,
                                                                                 norm_out, width);
  return launched("add_rmsnorm_kernel launch failed");
}

extern "C" int b2_swiglu(const uint16_t *gu, uint16_t *out, int32_t rows, int32_t ffn, void *stream) {
  if (rows < 0) return b2_record_error(B2_ERR_ARG, "b2_swiglu: rows must be >= 0");
  if (rows == 0) return b2_clear_error();
  if (!gu || !out) return b2_record_error(B2_ERR_ARG, "b2_swiglu: null pointer argument");
  if (ffn <= 0 || ffn % 8) return b2_record_error(B2_ERR_ARG, "b2_swiglu: ffn must be a positive multiple of 8");
  if (!aligned16(gu) || !aligned16(out)) return b2_record_error(B2_ERR_ARG, "b2_swiglu: pointers must be 16-byte aligned");
  const int64_t n = static_cast<int64_t>(rows) * (ffn / 8);
  const int threads = 256;
  const int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 0x7fffffff) return b2_record_error(B2_ERR_ARG, "b2_swiglu: too many rows");
  swiglu_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(gu, out, rows, ffn);
  return launched("swiglu_kernel launch failed");
}

extern "C" int b2_shortconv_step(const uint16_t *bcx, uint16_t *conv_state, const uint16_t *conv_w, uint16_t *out,
                                 int32_t rows, int32_t hidden, void *stream) {
  if (rows < 0) return b2_record_error(B2_ERR_ARG, "b2_shortconv_step: rows must be >= 0");
  if (rows == 0) return b2_clear_error();
  if (!bcx || !conv_state || !conv_w || !out)
    return b2_record_error(B2_ERR_ARG, "b2_shortconv_step: null pointer argument");
  if (hidden <= 0) return b2_record_error(B2_ERR_ARG, "b2_shortconv_step: hidden must be positive");
  if (rows > 65535) return b2_record_error(B2_ERR_ARG, "b2_shortconv_step: rows must be <= 65535");
  const int threads = 256;
  const dim3 grid((hidden + threads - 1) / threads, rows);
  shortconv_step_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(bcx, conv_state, conv_w, out, rows,
                                                                                hidden);
  return launched("shortconv_step_kernel launch failed");
}

extern "C" int b2_argmax_rows(const uint16_t *logits, int32_t rows, int32_t cols, int64_t *out, void *stream) {
  if (rows < 0) return b2_record_error(B2_ERR_ARG, "b2_argmax_rows: rows must be >= 0");
  if (rows == 0) return b2_clear_error();
  if (!logits || !out) return b2_record_error(B2_ERR_ARG, "b2_argmax_rows: null pointer argument");
  if (cols <= 0 || cols % 8) return b2_record_error(B2_ERR_ARG, "b2_argmax_rows: cols must be a positive multiple of 8");
  if (!aligned16(logits)) return b2_record_error(B2_ERR_ARG, "b2_argmax_rows: logits must be 16-byte aligned");
  argmax_rows_kernel<<<rows, kArgmaxThreads, 0, static_cast<cudaStream_t>(stream)>>>(logits, cols, out);
  return launched("argmax_rows_kernel launch failed");
}
