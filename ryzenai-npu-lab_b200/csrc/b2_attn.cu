// B200 (sm_100a) kernels and C ABI for LFM2.5 decode attention.
//
//   append_rope_kernel   q/k RMSNorm + rotate-half RoPE + paged KV append
//   paged_decode_kernel  split-KV flash-decode, TMA + mbarrier pipeline
//   combine_kernel       log-sum-exp merge of partial softmax states
//   decode_step_kernel   the whole decode step in one persistent launch
//                        (norm + RoPE + append + split-KV attention + merge)
//   prefill_attn_kernel  batched-prompt attention on tcgen05 (TMEM accumulators)
//
// Model constants: 16 query heads, 8 KV heads, head_dim 64, 64-token blocks.
// The numerics follow the reference's PyTorch BF16 path (Hugging Face
// transformers Lfm2Attention, modeling_lfm2.py: Lfm2RMSNorm.forward 59-64,
// apply_rotary_pos_emb 163-185, sdpa/eager attention 200-223), which is what
// the reference's fixtures were generated with (006_lfm25_baseline.py:115-117).

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "b2_decode_attn.h"
#include "b2_internal.h"

namespace {

constexpr int kHq = 16;
constexpr int kHkv = 8;
constexpr int kDim = 64;
constexpr int kBlock = 64;
constexpr int kQkvWidth = (kHq + 2 * kHkv) * kDim;  // 2048

// decode kernel geometry
constexpr int kStages = 4;
constexpr int kConsumerWarps = 4;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;
constexpr int kTileBytes = kBlock * kDim * 2;  // one (block, head) tile: 8 KiB
constexpr int kStageBytes = 2 * kTileBytes;    // K tile + V tile
// Default limit of a wait on another thread of the CTA (2 s), then the
// kernel reports B2_DEV_TIMEOUT and unwinds; b2_set_wait_limits changes it
// per process.  Waits for the CTA's own copies or tensor-core products (the
// hardware, not another thread) always allow kDrainLimitNs.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
constexpr uint64_t kDrainLimitNs = 2000000000ull;

struct __align__(8) DecodeTail {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  float red[kConsumerWarps][2][2 + kDim];
};
constexpr int kDecodeSmem = kStages * kStageBytes + 1024 + (int)sizeof(DecodeTail);

thread_local char g_err[512];

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = 0;
  return B2_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Widest block table (and largest split) accepted: width x 64 tokens must stay
// an int32 token count, which every length check on the device computes.
constexpr int32_t kMaxTableWidth = (1 << 25) - 1;

int table_width_error(int32_t max_blocks_per_seq) {
  return fail(B2_ERR_ARG, "max_blocks_per_seq must be <= %d (got %d)", kMaxTableWidth, max_blocks_per_seq);
}

// ------------------------------------------------------------------ device helpers

__device__ __forceinline__ void unpack8(const uint4 &w, float f[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}

// round-to-nearest-even fp32 -> bf16 bits (the rounding torch uses on CPU)
__device__ __forceinline__ uint32_t bf16_bits(float x) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(x)));
}

__device__ __forceinline__ float bf16_round(float x) {
  return __uint_as_float(bf16_bits(x) << 16);
}

// two fp32 -> one bf16x2 word (lo in the low half), round-to-nearest-even,
// in one paired conversion instruction
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ uint4 pack8(const float f[8]) {
  uint4 w;
  w.x = pack_bf16x2_rn(f[0], f[1]);
  w.y = pack_bf16x2_rn(f[2], f[3]);
  w.z = pack_bf16x2_rn(f[4], f[5]);
  w.w = pack_bf16x2_rn(f[6], f[7]);
  return w;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete; false after
// limit_ns (the caller reports B2_DEV_TIMEOUT and unwinds).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Expect `bytes` more of the current phase's transfer without arriving: the
// phase completes once the bytes have landed and the arrival comes later.
__device__ __forceinline__ void mbar_expect_tx_only(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// 2-D tiled TMA load into this CTA alone, completing on an mbarrier; KV tiles are
// read once per step, so they are marked evict-first in L2.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// ------------------------------------------------------------------ append + RoPE

struct AppendArgs {
  const uint16_t *qkv;
  int64_t row_stride;
  const uint16_t *gamma_q, *gamma_k;
  float eps;
  const uint16_t *cos, *sin;
  int rope_rows;
  const int32_t *past_lens;
  const int32_t *block_tables;
  int max_blocks;
  uint16_t *k_pool, *v_pool;
  int num_blocks;
  uint16_t *q_out;
  int mode;
  int32_t *err;
  int tokens;                 // tokens per sequence in qkv / q_out rows (1 for decode)
  const int32_t *chunk_lens;  // valid tokens per sequence (NULL: all `tokens`)
};

// Per-head RMSNorm (optional) and rotate-half RoPE (optional) of one 64-wide
// head vector spread over an aligned group of 8 lanes: chunk j = lane % 8
// holds x[8] = elements 8j..8j+7.  Every lane of the warp must call this
// (it shuffles with the full mask); `norm` / `rope` may differ per group.
//  * Lfm2RMSNorm: gamma * bf16(x * 1/sqrt(mean(x^2) + eps)) with fp32 math and
//    IEEE-rounded sqrt and divide, as torch's CPU rsqrt computes 1/sqrt.
//  * RoPE: bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)), rotate_half(x) =
//    [-x[32:], x[:32]]; the partner chunk j^4 sits on lane^4.
//
// mean(x^2) is bit-identical to torch's CPU x.pow(2).mean(-1) of a contiguous
// 64-float row: rounded squares, summed in the order of ATen's vectorised
// inner-dimension sum, whose vectors are 8 floats wide on every CPU build
// (the reduction is not dispatched to 16-wide vectors), then divided by 64
// (exact).  With v_k = squares 8k..8k+7 (chunk k, held by lane k of the group):
//   a_k = v_k + v_{k+4}              k = 0..3, lane-wise
//   p   = ((a_0 + a_1) + a_2) + a_3   lane-wise
//   sum = (((p[0] + p[1]) + p[2]) + ...) + p[7]
// No fused multiply-add anywhere in the chain.
__device__ __forceinline__ float sum_squares64(const float x[8]) {
  const int base = (threadIdx.x & 31) & ~7;
  float a[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float sq = __fmul_rn(x[e], x[e]);
    a[e] = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 4));  // a_k on lanes k = 0..3
  }
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a0 = __shfl_sync(0xffffffffu, a[e], base);
    const float a1 = __shfl_sync(0xffffffffu, a[e], base + 1);
    const float a2 = __shfl_sync(0xffffffffu, a[e], base + 2);
    const float a3 = __shfl_sync(0xffffffffu, a[e], base + 3);
    const float p = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
    s = e == 0 ? p : __fadd_rn(s, p);
  }
  return s;
}

__device__ __forceinline__ void norm_rope8_v(float x[8], int j, bool norm, bool rope, const uint4 gam,
                                             float eps, const uint4 cos8, const uint4 sin8) {
  const float ss = sum_squares64(x);
  if (norm) {
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss * (1.0f / kDim), eps)));
    float g[8];
    unpack8(gam, g);
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = bf16_round(__fmul_rn(g[e], bf16_round(__fmul_rn(x[e], inv))));
  }
  float p[8];
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const uint32_t w = bf16_bits(x[e]) | (bf16_bits(x[e + 1]) << 16);
    const uint32_t o = __shfl_xor_sync(0xffffffffu, w, 4);
    p[e] = __uint_as_float(o << 16);
    p[e + 1] = __uint_as_float(o & 0xffff0000u);
  }
  if (rope) {
    float c[8], s[8];
    unpack8(cos8, c);
    unpack8(sin8, s);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float rot = j < 4 ? -p[e] : p[e];
      const float part1 = bf16_round(__fmul_rn(x[e], c[e]));
      const float part2 = bf16_round(__fmul_rn(rot, s[e]));
      x[e] = bf16_round(__fadd_rn(part1, part2));
    }
  }
}

// The same with gamma (the 8 values at j * 8) and the RoPE rows read here.
__device__ __forceinline__ void norm_rope8(float x[8], int j, bool norm, bool rope,
                                           const uint16_t *gamma, float eps,
                                           const uint16_t *cos_row, const uint16_t *sin_row) {
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  norm_rope8_v(x, j, norm, rope, norm ? *reinterpret_cast<const uint4 *>(gamma + j * 8) : zero, eps,
               rope ? *reinterpret_cast<const uint4 *>(cos_row + j * 8) : zero,
               rope ? *reinterpret_cast<const uint4 *>(sin_row + j * 8) : zero);
}

// One CTA (8 warps) per token: grid (sequence, token of the chunk).  The 32
// head vectors of a qkv row (16 q, 8 k, 8 v) are split 4 per warp; 8 lanes
// own one vector, 8 consecutive bf16 (16 bytes) each, so loads and stores
// are 16-byte vectors and a vector's rotate-half partner chunk (d +- 32)
// sits on lane^4.  Token t of sequence b goes to position past_lens[b] + t.
__global__ void __launch_bounds__(256) append_rope_kernel(const AppendArgs a) {
  const int b = blockIdx.x;
  const int tok = blockIdx.y;
  if (a.chunk_lens && tok >= a.chunk_lens[b]) return;
  const int64_t row = (int64_t)b * a.tokens + tok;
  const int lane = threadIdx.x & 31;
  const int vec = (threadIdx.x >> 5) * 4 + (lane >> 3);  // 0..31
  const int j = lane & 7;                                // 16-byte chunk
  const bool is_q = vec < kHq;
  const bool is_v = vec >= kHq + kHkv;
  const int pos = a.past_lens[b] + tok;

  float x[8];
  unpack8(*reinterpret_cast<const uint4 *>(a.qkv + row * a.row_stride + vec * kDim + j * 8), x);
  const bool pos_ok = pos >= 0 && pos < a.max_blocks * kBlock;
  const bool rope_ok = pos >= 0 && pos < a.rope_rows;
  if ((a.mode & B2_ROPE_QK) && !rope_ok && j == 0 && vec == 0) atomicOr(a.err, B2_DEV_BAD_POSITION);
  const bool rope = !is_v && (a.mode & B2_ROPE_QK) && rope_ok;
  norm_rope8(x, j, !is_v && (a.mode & B2_NORM_QK), rope, is_q ? a.gamma_q : a.gamma_k, a.eps,
             rope ? a.cos + (int64_t)pos * kDim : nullptr, rope ? a.sin + (int64_t)pos * kDim : nullptr);

  if (is_q) {
    if (a.q_out)
      *reinterpret_cast<uint4 *>(a.q_out + (row * kHq + vec) * kDim + j * 8) = pack8(x);
    return;
  }
  if (!(a.mode & B2_STORE_KV)) return;
  if (!pos_ok) {
    if (j == 0 && vec == kHq) atomicOr(a.err, B2_DEV_BAD_LENGTH);
    return;
  }
  const int blk = a.block_tables[(int64_t)b * a.max_blocks + pos / kBlock];
  if (blk < 0 || blk >= a.num_blocks) {
    if (j == 0 && vec == kHq) atomicOr(a.err, B2_DEV_BAD_BLOCK);
    return;
  }
  const int head = is_v ? vec - kHq - kHkv : vec - kHq;
  const int64_t off = (((int64_t)blk * kHkv + head) * kBlock + (pos % kBlock)) * kDim + j * 8;
  *reinterpret_cast<uint4 *>((is_v ? a.v_pool : a.k_pool) + off) = pack8(x);
}

// ------------------------------------------------------------------ split-KV decode

struct DecodeArgs {
  const uint16_t *q;
  const int32_t *block_tables;
  int max_blocks;
  const int32_t *seq_lens;
  int num_blocks;
  int blocks_per_split;
  int num_splits;
  float scale_log2;
  float *part_ml;
  float *part_o;
  int32_t *err;
  uint64_t wait_ns;  // limit of a wait on another warp
};

// grid (num_splits, 8 kv heads, batch), 4 consumer warps + 1 producer warp.
//
// Producer (warp 4, lane 0): for each 64-token block of the split, TMA-loads
// the K and V tiles of this KV head (8 KiB each, rows swizzled in 128-byte
// groups) into a ring of kStages stages, each guarded by a full/empty
// mbarrier pair.
//
// Consumers: warp w owns rows [16w, 16w+16) of every tile and keeps its own
// online-softmax state (running max m and sum l per query head, log2 units).
//  * q.K: lane (r = lane/2, half = lane%2) dots 32 dims of row r with both
//    query heads (2kv, 2kv+1) and the pair is summed by one shuffle.
//  * p.V: lane (c = lane%8, g = lane/8) accumulates 8 dims (chunk c) of rows
//    4g..4g+3 for both heads in 16 fp32 registers.
// The 128-byte swizzle makes both access patterns bank-conflict free.
// Warps and lanes are merged once per CTA into the partial state.
__global__ void __launch_bounds__(kDecodeThreads, 3)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const DecodeArgs a) {
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;
  const int b = blockIdx.z;
  const int seq_len = a.seq_lens[b];
  if (seq_len < 0 || seq_len > a.max_blocks * kBlock) {
    if (threadIdx.x == 0 && split == 0 && kvh == 0) atomicOr(a.err, B2_DEV_BAD_LENGTH);
    return;
  }
  const int nblk = (seq_len + kBlock - 1) / kBlock;
  const int b0 = split * a.blocks_per_split;
  const int b1 = min(nblk, b0 + a.blocks_per_split);
  if (b0 >= b1) return;  // this split lies past the end of the sequence
  const int n = b1 - b0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *tiles = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  DecodeTail *tail = reinterpret_cast<DecodeTail *>(tiles + kStages * kStageBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&tail->full[s]), 1);
      mbar_init(smem_u32(&tail->empty[s]), kConsumerWarps);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane != 0) return;
    // ---------------- producer
    const uint64_t policy = evict_first_policy();
    const int32_t *tbl = a.block_tables + (int64_t)b * a.max_blocks + b0;
    int issued = 0;
    for (int i = 0; i < n; ++i) {
      const int s = i % kStages;
      const uint32_t ph = (i / kStages) & 1;
      if (i >= kStages && !mbar_wait(smem_u32(&tail->empty[s]), ph ^ 1, a.wait_ns)) {
        atomicOr(a.err, B2_DEV_TIMEOUT);
        break;
      }
      int blk = tbl[i];
      if (blk < 0 || blk >= a.num_blocks) {
        atomicOr(a.err, B2_DEV_BAD_BLOCK);
        blk = 0;  // read a valid tile instead; the result is flagged as bad
      }
      const int row = (blk * kHkv + kvh) * kBlock;
      const uint32_t full = smem_u32(&tail->full[s]);
      uint8_t *dst = tiles + s * kStageBytes;
      mbar_expect_tx(full, kStageBytes);
      tma_load_2d(smem_u32(dst), &tm_k, 0, row, full, policy);
      tma_load_2d(smem_u32(dst + kTileBytes), &tm_v, 0, row, full, policy);
      issued = i + 1;
    }
    // Do not leave while a copy into this CTA's shared memory is in flight:
    // wait (bounded) for the last phase issued on every stage.
    for (int s = 0; s < kStages && s < issued; ++s) {
      const int last = s + kStages * ((issued - 1 - s) / kStages);
      if (!mbar_wait(smem_u32(&tail->full[s]), (last / kStages) & 1, kDrainLimitNs))
        atomicOr(a.err, B2_DEV_TIMEOUT);
    }
    return;
  }

  // ---------------- consumers
  const int r = lane >> 1, half = lane & 1;  // q.K mapping
  const int c = lane & 7, g = lane >> 3;     // p.V mapping
  float q0[32], q1[32];
  {
    const uint16_t *qb = a.q + ((int64_t)b * kHq + 2 * kvh) * kDim + half * 32;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      unpack8(*reinterpret_cast<const uint4 *>(qb + k * 8), q0 + k * 8);
      unpack8(*reinterpret_cast<const uint4 *>(qb + kDim + k * 8), q1 + k * 8);
    }
  }
  float m0 = -1.0e30f, m1 = -1.0e30f;  // finite floor: exp2 of (floor - floor) stays 1
  float lsum = 0.f;                    // this lane's sum for head `half`
  float acc0[8], acc1[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc0[e] = acc1[e] = 0.f;

  const int qrow = 16 * warp + r;
  for (int i = 0; i < n; ++i) {
    const int s = i % kStages;
    const uint32_t ph = (i / kStages) & 1;
    if (!mbar_wait(smem_u32(&tail->full[s]), ph, a.wait_ns)) {
      if (lane == 0) atomicOr(a.err, B2_DEV_TIMEOUT);
      break;
    }
    const uint8_t *kt = tiles + s * kStageBytes;
    const uint8_t *vt = kt + kTileBytes;
    const int valid = seq_len - ((b0 + i) * kBlock + 16 * warp);  // valid rows of this warp

    float d0 = 0.f, d1 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int pc = (half * 4 + k) ^ (qrow & 7);
      float f[8];
      unpack8(*reinterpret_cast<const uint4 *>(kt + qrow * 128 + pc * 16), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d0 = fmaf(q0[k * 8 + e], f[e], d0);
        d1 = fmaf(q1[k * 8 + e], f[e], d1);
      }
    }
    d0 += __shfl_xor_sync(0xffffffffu, d0, 1);
    d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
    const bool tv = r < valid;
    const float s0 = tv ? d0 * a.scale_log2 : -INFINITY;
    const float s1 = tv ? d1 * a.scale_log2 : -INFINITY;
    float bm0 = s0, bm1 = s1;
#pragma unroll
    for (int off = 2; off < 32; off <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
    }
    const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
    const float a0 = ex2(m0 - mn0), a1 = ex2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const float p = ex2((half ? s1 : s0) - (half ? mn1 : mn0));  // 0 for masked rows
    lsum = fmaf(lsum, half ? a1 : a0, p);

#pragma unroll
    for (int e = 0; e < 8; ++e) {
      acc0[e] *= a0;
      acc1[e] *= a1;
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int t = 4 * g + jj;
      const float p0 = __shfl_sync(0xffffffffu, p, 2 * t);
      const float p1 = __shfl_sync(0xffffffffu, p, 2 * t + 1);
      if (t < valid) {
        const int vrow = 16 * warp + t;
        float f[8];
        unpack8(*reinterpret_cast<const uint4 *>(vt + vrow * 128 + ((c ^ (vrow & 7)) * 16)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          acc0[e] = fmaf(p0, f[e], acc0[e]);
          acc1[e] = fmaf(p1, f[e], acc1[e]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&tail->empty[s]));
  }

  // ---------------- merge lanes, then warps
#pragma unroll
  for (int off = 2; off < 32; off <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    acc0[e] += __shfl_xor_sync(0xffffffffu, acc0[e], 8);
    acc0[e] += __shfl_xor_sync(0xffffffffu, acc0[e], 16);
    acc1[e] += __shfl_xor_sync(0xffffffffu, acc1[e], 8);
    acc1[e] += __shfl_xor_sync(0xffffffffu, acc1[e], 16);
  }
  if (lane < 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      tail->red[warp][0][2 + c * 8 + e] = acc0[e];
      tail->red[warp][1][2 + c * 8 + e] = acc1[e];
    }
  }
  if (lane < 2) {
    tail->red[warp][lane][0] = lane ? m1 : m0;
    tail->red[warp][lane][1] = lsum;
  }
  consumer_bar();
  const int h = threadIdx.x >> 6;  // 0..1
  const int d = threadIdx.x & 63;
  float M = -1.0e30f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, tail->red[w][h][0]);
  float L = 0.f, O = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    const float sc = ex2(tail->red[w][h][0] - M);
    L = fmaf(tail->red[w][h][1], sc, L);
    O = fmaf(tail->red[w][h][2 + d], sc, O);
  }
  const int64_t idx = ((int64_t)b * a.num_splits + split) * kHq + 2 * kvh + h;
  a.part_o[idx * kDim + d] = O;
  if (d == 0) {
    a.part_ml[idx * 2] = M;
    a.part_ml[idx * 2 + 1] = L;
  }
}


// ------------------------------------------------------------------ multi-GPU state exchange (NVLink P2P)

// One sequence's KV cache split along the token axis over `world` GPUs: every
// rank holds a partial softmax state (max, sum, unnormalised output) per
// (sequence, query head).  Instead of an all-gather collective followed by a
// merge launch, one kernel writes this rank's state straight into every
// rank's exchange area over NVLink (peer pointers from CUDA IPC) and merges
// the world's states once they have arrived in its own area.
//
// Every value travels as one 8-byte word {float bits, tag}, written with a
// single 8-byte store, where tag = step number + 1 (the low-latency protocol
// of collective libraries): a reader polls the words themselves until their
// tags show the current step, so no fence or separate flag is needed.
// Exchange area (every rank, same layout; zeroed before first use):
//   uint2 word[2 slots][world][batch][16][kXState]   (m, l, 2 unused, o[64])
//   int   step[batch][16]                            (local step counter)
// Steps alternate slots.  A rank can be at most one step ahead of another
// (its next merge needs the other's words of that step, written after the
// other's previous merge finished reading), so a slot is never overwritten
// while it is read.

constexpr int kXState = 4 + kDim;
constexpr int kXMaxWorld = B2_XCHG_MAX_WORLD;
constexpr uint64_t kXWaitNs = 5000000000ull;  // default poll limit (5 s), then B2_DEV_TIMEOUT

struct XchgArgs {
  const float *state_ml;  // [batch][16][2]
  const float *state_o;   // [batch][16][64]
  int batch, world, rank;
  uint16_t *out;  // [batch][16][64]
  int32_t *err;
  char *area[kXMaxWorld];  // rank r's exchange area as mapped on this GPU
  uint64_t poll_ns;        // limit of the poll for the other ranks' words
};

__host__ __device__ constexpr int64_t x_words(int world, int batch) {
  return 2ll * world * batch * kHq * kXState;
}

__device__ __forceinline__ void st_word(uint2 *p, float v, uint32_t tag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag)
               : "memory");
}

__device__ __forceinline__ uint2 ld_word(const uint2 *p) {
  uint2 w;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(w.x), "=r"(w.y) : "l"(p) : "memory");
  return w;
}


// Exchange this rank's state (m, l, o[d] of thread d) for (sequence b, query
// head h) with every rank and write the world-merged context.  Run by 64
// threads (d = 0..63) that can sync on named barrier 2; see the exchange
// area layout above.
__device__ __forceinline__ void xchg_merge(const XchgArgs &a, int b, int h, int d, float m, float l, float o) {
  const int bh = b * kHq + h;
  const uint2 *own = reinterpret_cast<const uint2 *>(a.area[a.rank]);
  int32_t *steps = reinterpret_cast<int32_t *>(reinterpret_cast<uint2 *>(a.area[a.rank]) + x_words(a.world, a.batch));
  const int32_t step = steps[bh];
  const int slot = step & 1;
  const uint32_t tag = static_cast<uint32_t>(step) + 1u;
  const int64_t mine = (((static_cast<int64_t>(slot) * a.world + a.rank) * a.batch + b) * kHq + h) * kXState;
  for (int r = 0; r < a.world; ++r) {
    uint2 *dst = reinterpret_cast<uint2 *>(a.area[r]) + mine;
    st_word(dst + 4 + d, o, tag);
    if (d == 0) {
      st_word(dst, m, tag);
      st_word(dst + 1, l, tag);
    }
  }
  float M = -1.0e30f, L = 0.f, O = 0.f;
  bool ok = true;
  const uint64_t t0 = global_ns();
  for (int r = 0; r < a.world && ok; ++r) {
    const uint2 *src = own + (((static_cast<int64_t>(slot) * a.world + r) * a.batch + b) * kHq + h) * kXState;
    uint2 wm, wl, wo;
    for (;;) {
      wm = ld_word(src);
      wl = ld_word(src + 1);
      wo = ld_word(src + 4 + d);
      if (wm.y == tag && wl.y == tag && wo.y == tag) break;
      if (global_ns() - t0 > a.poll_ns) {
        atomicOr(a.err, B2_DEV_TIMEOUT);
        ok = false;
        break;
      }
    }
    if (!ok) break;
    const float ms = __uint_as_float(wm.x), ls = __uint_as_float(wl.x), os = __uint_as_float(wo.x);
    const float nm = fmaxf(M, ms);
    const float c1 = ex2(M - nm), c2 = ex2(ms - nm);
    L = L * c1 + ls * c2;
    O = O * c1 + os * c2;
    M = nm;
  }
  if (ok) a.out[(int64_t)bh * kDim + d] = static_cast<uint16_t>(bf16_bits(L > 0.f ? O / L : 0.f));
  asm volatile("bar.sync 2, 64;" ::: "memory");  // every thread has read its words of this step
  if (d == 0) steps[bh] = step + 1;
}

// ------------------------------------------------------------------ combine

struct CombineArgs {
  const float *part_ml;
  const float *part_o;
  int num_parts;
  const int32_t *seq_lens;
  int blocks_per_split;
  uint16_t *out;
  float *state_ml;
  float *state_o;
  int len_offset;   // 1 when seq_lens holds past lengths (the new token is added)
  int skip_single;  // sequences with one part were written by the decode kernel
  int max_tokens;   // num_parts * blocks_per_split * 64: longer lengths are invalid
  // float strides between sequences (b) and parts (s); 0 = the default
  // [batch][num_parts][16][2 | 64] layout
  int64_t ml_b, ml_s, o_b, o_s;
  int groups;  // part groups per CTA (blockDim.x / 64), 1..8
  XchgArgs x;  // x.world > 0: exchange the merged state with the other ranks (out = x.out)
};

// Part groups for a merge of up to num_parts parts: enough threads to merge
// hundreds of parts quickly, few for the usual handful (small CTAs launch fast).
// At most 8 groups (512 threads): a CTA of that size still fits beside the
// decode-step CTAs, so it can launch early as a programmatic dependent.
int combine_groups(int num_parts) {
  int g = 1;
  while (g < 8 && g * 4 < num_parts) g *= 2;
  return g;
}

// grid (batch, 16 heads), block (groups x 64 dims).  Group g merges parts
// g, g + groups, ... with a running (max, sum, output), loading four parts
// per round; the group states are then merged in shared memory, so a
// sequence split into hundreds of parts is still merged by many threads.
// With an exchange (a.x.world > 0) group 0 then runs xchg_merge with the
// merged state instead of writing it.
// When launched as a programmatic dependent of the decode-step kernel it may
// start early; griddepcontrol.wait holds it until that kernel has completed
// and its memory is visible (a no-op for an ordinary launch).
constexpr int kCombineGroups = 16;  // upper bound of the arrays; combine_groups() uses at most 8

__global__ void __launch_bounds__(kCombineGroups * kDim) combine_kernel(const CombineArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float sm[kCombineGroups], sl[kCombineGroups], so[kCombineGroups][kDim];
  const int b = blockIdx.x;
  const int h = blockIdx.y;
  const int grp = threadIdx.x >> 6;
  const int d = threadIdx.x & 63;
  const bool exchange = a.x.world > 0;
  int parts = a.num_parts;
  if (a.seq_lens) {
    const int len = a.seq_lens[b] + a.len_offset;
    // an invalid length (flagged by the decode kernel) still takes part in an
    // exchange, with an empty state, so that no rank waits for it in vain
    if (len > a.max_tokens && !exchange) return;
    const int nblk = len > 0 && len <= a.max_tokens ? (len + kBlock - 1) / kBlock : 0;
    parts = min(parts, (nblk + a.blocks_per_split - 1) / a.blocks_per_split);
    if (a.skip_single && parts == 1 && !exchange) return;  // written by the decode kernel
  }
  const int64_t ml_s = a.ml_s ? a.ml_s : kHq * 2;
  const int64_t ml_b = a.ml_b ? a.ml_b : a.num_parts * ml_s;
  const int64_t o_s = a.o_s ? a.o_s : kHq * kDim;
  const int64_t o_b = a.o_b ? a.o_b : a.num_parts * o_s;
  const float *ml = a.part_ml + b * ml_b + h * 2;
  const float *po = a.part_o + b * o_b + h * kDim + d;
  float M = -1.0e30f, L = 0.f, O = 0.f;
  // four parts per group and round: their loads are issued together
  for (int s0 = grp; s0 < parts; s0 += 4 * a.groups) {
    float mv[4], lv[4], ov[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int s = s0 + k * a.groups;
      const bool in = s < parts;
      mv[k] = in ? ml[s * ml_s] : -1.0e30f;
      lv[k] = in ? ml[s * ml_s + 1] : 0.f;
      ov[k] = in ? po[s * o_s] : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float nm = fmaxf(M, mv[k]);
      const float c1 = ex2(M - nm), c2 = ex2(mv[k] - nm);
      L = L * c1 + lv[k] * c2;
      O = O * c1 + ov[k] * c2;
      M = nm;
    }
  }
  if (d == 0) {
    sm[grp] = M;
    sl[grp] = L;
  }
  so[grp][d] = O;
  __syncthreads();
  if (grp != 0) return;
  float MM = -1.0e30f;
  for (int g = 0; g < a.groups; ++g) MM = fmaxf(MM, sm[g]);
  float LL = 0.f, OO = 0.f;
  for (int g = 0; g < a.groups; ++g) {
    const float c = ex2(sm[g] - MM);
    LL = fmaf(sl[g], c, LL);
    OO = fmaf(so[g][d], c, OO);
  }
  if (exchange) {
    xchg_merge(a.x, b, h, d, MM, LL, OO);  // this rank's merged state to every rank; world merge
    return;
  }
  const int64_t oi = ((int64_t)b * kHq + h) * kDim + d;
  if (a.out) a.out[oi] = static_cast<uint16_t>(bf16_bits(LL > 0.f ? OO / LL : 0.f));
  if (a.state_o) {
    a.state_o[oi] = OO;
    if (d == 0) {
      a.state_ml[((int64_t)b * kHq + h) * 2] = MM;
      a.state_ml[((int64_t)b * kHq + h) * 2 + 1] = LL;
    }
  }
}

// ------------------------------------------------------------------ fused persistent decode step

// One launch per decode step: q/k norm + RoPE + KV append + split-KV
// attention + merge.  A persistent grid (3 CTAs per SM) takes work items
// (split, sequence, kv head) from a global counter; the producer warp keeps
// the TMA ring full across item boundaries, so the pipeline never drains
// between items and the end-of-launch tail is at most one short item per CTA.
constexpr int kFlagFirst = 1;  // first block of an item: load q, reset state
constexpr int kFlagLast = 2;   // last block of an item: epilogue
constexpr int kFlagFinal = 4;  // the item is the whole sequence: write the context directly
constexpr int kFlagEnd = 8;    // no more work

// kT: the largest number of new tokens per sequence of the instantiation (1,
// or 4 for b2_decode_step_tokens).
template <int kT>
struct __align__(16) StageMetaT {
  int b, kvh, split, rows;   // rows: valid rows of this block for the item's last token (may exceed 64)
  int flags, nsplit, ntok, pad1;  // ntok: new tokens of the sequence (1 when kT == 1)
  uint16_t q[kT * 2 * kDim];  // bf16 q [token][head 2kvh, 2kvh+1][64] (first block of an item)
};

// Batches up to this size enumerate only real work items: the producer
// warp builds the prefix sum of splits per sequence in shared memory at start.
// Larger batches walk the dense (split, sequence, head) space and skip the
// splits that lie past a sequence's end.
constexpr int kMaxCompactBatch = 512;

// Warps of the fused kernel: 4 consumers, 1 producer (TMA), 1 merger (the
// cross-CTA arrival count and the merge of a sequence's splits, off the
// consumers' path).
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kMergerWarp = kConsumerWarps + 1;
constexpr int kStepThreads = (kConsumerWarps + 2) * 32;
constexpr int kPubSlots = 4;  // items published to the merger warp, in flight
constexpr int kMergeInKernelSplits = 16;  // at most 32: one split per merger lane
constexpr int kMaxStepTokens = 4;  // new tokens per sequence of b2_decode_step_tokens (N = 8 mma columns / 2 heads)
constexpr int kStepMaxBlocksPerSplit = 64;  // two block-table entries per producer lane

template <int kT>
struct __align__(16) StepTailT {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t ebar;  // consumer-warp barrier of the epilogue (bounded waits)
  uint64_t stall;  // never completed: the wait of B2_TEST_STALL runs out on it
  uint64_t pub[kPubSlots];    // consumers -> merger: a partial state is in memory
  uint64_t pfree[kPubSlots];  // merger -> consumers: the slot may be reused
  int4 pubinfo[kPubSlots];    // (b, kv head, split or new tokens, nsplit); b < 0 ends the work
  StageMetaT<kT> meta[kStages];
  float red[2][kConsumerWarps][2 * kT][2 + kDim];  // double-buffered by epilogue parity; [token][head]
  int prefix[kMaxCompactBatch + 1];  // prefix[b] = splits of sequences 0..b-1
};
template <int kT>
constexpr int step_smem() { return kStages * kStageBytes + 1024 + (int)sizeof(StepTailT<kT>); }
// CTAs per SM: 3 with one token (74 KB of shared memory each), 2 with up to 4
template <int kT>
constexpr int step_ctas_per_sm() { return kT == 1 ? 3 : 2; }

struct StepArgs {
  const uint16_t *qkv;
  int64_t row_stride;
  const uint16_t *gamma_q, *gamma_k;
  float eps;
  const uint16_t *cos, *sin;
  int rope_rows;
  const int32_t *past_lens;
  const int32_t *seq_lens;  // tokens attended; NULL: past_lens + 1
  const int32_t *block_tables;
  int max_blocks;
  uint16_t *k_pool, *v_pool;
  int num_blocks;
  int batch, blocks_per_split, num_splits, total_items;
  int direct_out;  // whole-sequence items write the bf16 context themselves
  int merge_here;  // the merger warp merges the splits (else a combine kernel follows)
  float scale_log2;
  int mode;
  uint16_t *out, *q_out;
  float *state_ml, *state_o;  // merged fp32 state instead of out (direct_out == 0)
  float *part_ml, *part_o;
  int32_t *counters;  // [0] work counter, [1] finished CTAs, [2 + b * 8 + kv head] split arrivals
  int32_t *err;
  uint64_t wait_ns;  // limit of a wait on another warp
  // b2_decode_step_tokens: up to `tokens` new tokens per sequence (rows b *
  // tokens + t of qkv; chunk_lens[b] of them valid, all when NULL); contexts,
  // q_out and partial states gain a token index after the sequence's
  int tokens;
  const int32_t *chunk_lens;
};

// Barrier of the 4 consumer warps on an mbarrier, with a bounded wait (a
// hardware named barrier could not give up if a warp had left on a timeout).
template <class Tail>
__device__ __forceinline__ void consumers_sync(Tail *tail, int lane, uint32_t &phase, int32_t *err,
                                               uint64_t limit_ns) {
  __syncwarp();
  if (lane == 0) mbar_arrive(smem_u32(&tail->ebar));
  const bool ok = mbar_wait(smem_u32(&tail->ebar), phase & 1, limit_ns);
  ++phase;
  if (!ok && lane == 0) atomicOr(err, B2_DEV_TIMEOUT);
  __syncwarp();
}

// A 4-byte load from read-only memory, issued where it stands: the compiler
// may not move it next to its first use, so a run of these is in flight
// together.
__device__ __forceinline__ int ld_nc_now(const int *p) {
  int v;
  asm volatile("ld.global.nc.b32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Lengths of sequence b: past (RoPE position and, with B2_STORE_KV, the
// append slot) and seq_len (tokens attended).  False for lengths the block
// table cannot hold, or an append slot that is not the last attended token.
__device__ __forceinline__ bool lengths_ok(const StepArgs &a, int past, int seq_len) {
  bool ok = past >= 0 && seq_len >= 0 && seq_len <= a.max_blocks * kBlock;
  if (a.mode & B2_STORE_KV) ok = ok && seq_len == past + 1;
  return ok;
}

// Several new tokens (kT > 1): the chunk of sequence b is chunk_lens[b]
// (all `tokens` when NULL), its tokens sit at past .. past + chunk - 1, and the
// last of them attends past + chunk tokens.
__device__ __forceinline__ bool chunk_ok(const StepArgs &a, int past, int chunk) {
  return past >= 0 && chunk >= 1 && chunk <= a.tokens &&
         static_cast<int64_t>(past) + chunk <= static_cast<int64_t>(a.max_blocks) * kBlock;
}

template <int kT>
__device__ __forceinline__ bool step_lengths(const StepArgs &a, int b, int &past, int &seq_len, int &ntok) {
  past = __ldg(a.past_lens + b);
  if constexpr (kT == 1) {
    ntok = 1;
    seq_len = a.seq_lens ? __ldg(a.seq_lens + b) : past + 1;
    return lengths_ok(a, past, seq_len);
  } else {
    ntok = a.chunk_lens ? __ldg(a.chunk_lens + b) : a.tokens;
    seq_len = past + ntok;
    return chunk_ok(a, past, ntok);
  }
}

// Empty result of sequence e (nothing to attend): a zero context, or the
// state (-inf, 0, 0).  One warp.
__device__ __forceinline__ void write_empty_result(const StepArgs &a, int e, int lane) {
  for (int i = lane; i < kHq * kDim; i += 32) {
    if (a.direct_out) a.out[(int64_t)e * kHq * kDim + i] = 0;
    else if (a.state_o) a.state_o[(int64_t)e * kHq * kDim + i] = 0.f;
  }
  if (!a.direct_out && a.state_ml && lane < kHq) {
    a.state_ml[((int64_t)e * kHq + lane) * 2] = -1.0e30f;
    a.state_ml[((int64_t)e * kHq + lane) * 2 + 1] = 0.f;
  }
}

// One work item as the producer sees it, with its loads already issued.
template <int kT>
struct ProducerItem {
  int valid, b, kvh, split, past, seq_len, nsplit, blk0, n, ntok;
  int my_blk;   // block table entry blk0 + lane (lane < n); entries from 32 on are read when needed
  uint4 raw[kT];  // this lane's 16 bytes of the item's q/k/v vectors, per new token
};

// Decode work index w and issue its loads.  Compact enumeration: w = p * 8 +
// kvh over the real (sequence, split) pairs p; dense: w = (split * batch + b)
// * 8 + kvh, returning valid = 0 for a split past the sequence's end (the
// caller skips it) and -1 past the end of the work.
template <int kT>
__device__ __forceinline__ ProducerItem<kT> producer_load(const StepArgs &a, const StepTailT<kT> *tail, bool compact,
                                                          int total, int w, int lane) {
  ProducerItem<kT> it;
  it.valid = -1;
  if (w >= total) return it;
  it.valid = 1;
  it.kvh = w & 7;
  const int p = w >> 3;
  if (compact) {
    int lo = 0, hi = a.batch;  // largest b with prefix[b] <= p
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (tail->prefix[mid] <= p) lo = mid; else hi = mid;
    }
    it.b = lo;
    it.split = p - tail->prefix[lo];
  } else {
    it.split = p / a.batch;
    it.b = p - it.split * a.batch;
  }
  const bool len_ok = step_lengths<kT>(a, it.b, it.past, it.seq_len, it.ntok);
  const int nblk = (it.seq_len + kBlock - 1) / kBlock;
  it.nsplit = (nblk + a.blocks_per_split - 1) / a.blocks_per_split;
  if (!len_ok || it.split >= it.nsplit) {
    if (!len_ok && lane == 0 && it.kvh == 0 && it.split == 0) atomicOr(a.err, B2_DEV_BAD_LENGTH);
    it.valid = 0;
    return it;
  }
  it.blk0 = it.split * a.blocks_per_split;
  it.n = min(a.blocks_per_split, nblk - it.blk0);
  it.my_blk = lane < it.n ? __ldg(a.block_tables + (int64_t)it.b * a.max_blocks + it.blk0 + lane) : 0;
  const int grp = lane >> 3;
  const int vec = grp < 2 ? 2 * it.kvh + grp : (grp == 2 ? kHq + it.kvh : kHq + kHkv + it.kvh);
  if constexpr (kT == 1) {
    it.raw[0] = __ldg(reinterpret_cast<const uint4 *>(a.qkv + it.b * a.row_stride + vec * kDim + (lane & 7) * 8));
  } else {
#pragma unroll
    for (int t = 0; t < kT; ++t)
      if (t < it.ntok)
        it.raw[t] = __ldg(reinterpret_cast<const uint4 *>(a.qkv + ((int64_t)it.b * a.tokens + t) * a.row_stride +
                                                          vec * kDim + (lane & 7) * 8));
  }
  return it;
}

// Producer warp: takes items from the work counter one ahead of the item it
// is issuing (the next item's counter update and loads are in flight while
// this item's copies wait for free stages), prepares q (and the appended k/v
// on the item holding the new token) with all 32 lanes, and lane 0 issues
// the TMA loads.  Lanes 0-15 hold the two q heads, 16-23 k, 24-31 v.
template <int kT>
__device__ __forceinline__ void step_producer(const StepArgs &a, StepTailT<kT> *tail, uint8_t *tiles,
                                              const CUtensorMap *tm_k, const CUtensorMap *tm_v,
                                              int lane) {
  int32_t *work_ctr = a.counters;
  const uint64_t policy = evict_first_policy();
  const int grp = lane >> 3, j = lane & 7;
  // With one split per sequence the dense enumeration has no split past a
  // sequence's end, so the compact one (and its prefix scan) is not needed.
  const bool compact = a.batch <= kMaxCompactBatch && a.num_splits > 1;
  int total = a.total_items;
  constexpr int kChunks = kMaxCompactBatch / 32;  // 32-sequence chunks of the largest compact batch
  if (compact) {
    // prefix[b + 1] = sum of splits of sequences 0..b.  Every lane loads the
    // lengths of its sequences (b = 32 k + lane) first, so that all the loads
    // are in flight together (one round trip for any batch), then the 32-wide
    // chunks are scanned in turn; CTA 0 also writes the empty results of the
    // sequences with nothing to attend (they get no work item).  (Measured: a
    // lane-owned run per lane and one scan of the run totals was ~1 us slower
    // for batches of 8-64.)
    int pl[kChunks], sl[kChunks];
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      if (32 * k < a.batch) {
        const int b = min(32 * k + lane, a.batch - 1);
        pl[k] = ld_nc_now(a.past_lens + b);
        if constexpr (kT == 1)
          sl[k] = a.seq_lens ? ld_nc_now(a.seq_lens + b) : 0;
        else  // the chunk; the sequence attends past + chunk tokens
          sl[k] = a.chunk_lens ? ld_nc_now(a.chunk_lens + b) : a.tokens;
      }
    }
    int running = 0;
#pragma unroll
    for (int k = 0; k < kChunks; ++k) {
      if (32 * k >= a.batch) break;
      const int b = 32 * k + lane;
      int ns = 0;
      bool empty = false;
      if (b < a.batch) {
        bool len_ok;
        if constexpr (kT == 1) {
          if (!a.seq_lens) sl[k] = pl[k] + 1;
          len_ok = lengths_ok(a, pl[k], sl[k]);
        } else {
          len_ok = chunk_ok(a, pl[k], sl[k]);
          sl[k] += pl[k];
        }
        if (len_ok) {
          const int nblk = (sl[k] + kBlock - 1) / kBlock;
          ns = (nblk + a.blocks_per_split - 1) / a.blocks_per_split;
          empty = sl[k] == 0;
        } else if (blockIdx.x == 0) {
          atomicOr(a.err, B2_DEV_BAD_LENGTH);
        }
      }
      int incl = ns;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      if (b < a.batch) tail->prefix[b + 1] = running + incl;
      running += __shfl_sync(0xffffffffu, incl, 31);
      if (blockIdx.x == 0) {
        unsigned mask = __ballot_sync(0xffffffffu, empty);
        while (mask) {
          const int e = 32 * k + __ffs(mask) - 1;
          mask &= mask - 1;
          write_empty_result(a, e, lane);
        }
      }
    }
    if (lane == 0) tail->prefix[0] = 0;
    __syncwarp();
    total = running * kHkv;
  } else if (kT == 1 && blockIdx.x == 0) {
    // Sequences with nothing to attend (seq_lens[b] == 0) get no work item:
    // write their empty result here.  The lengths of 32 * kChunks sequences
    // are loaded before any is examined.  (With new tokens every sequence
    // attends at least one.)
    for (int c0 = 0; c0 < a.batch; c0 += 32 * kChunks) {
      int pl[kChunks], sl[kChunks];
#pragma unroll
      for (int k = 0; k < kChunks; ++k) {
        const int b = min(c0 + 32 * k + lane, a.batch - 1);
        pl[k] = ld_nc_now(a.past_lens + b);
        sl[k] = a.seq_lens ? ld_nc_now(a.seq_lens + b) : pl[k] + 1;
      }
#pragma unroll
      for (int k = 0; k < kChunks; ++k) {
        const int b = c0 + 32 * k + lane;
        const bool empty = b < a.batch && lengths_ok(a, pl[k], sl[k]) && sl[k] == 0;
        unsigned mask = __ballot_sync(0xffffffffu, empty);
        while (mask) {
          const int e = c0 + 32 * k + __ffs(mask) - 1;
          mask &= mask - 1;
          write_empty_result(a, e, lane);
        }
      }
    }
  }
  int issued = 0;
  bool ok = true;
  const bool norm = grp < 3 && (a.mode & B2_NORM_QK);
  // Item w = blockIdx.x is this CTA's first (no counter round trip before the
  // first copies); the counter hands out gridDim.x, gridDim.x + 1, ... after it.
  bool first_claim = true;
  auto next_item = [&]() {
    ProducerItem<kT> it;
    do {
      int w = 0;
      if (first_claim) {
        w = blockIdx.x;
        first_claim = false;
      } else {
        if (lane == 0) w = atomicAdd(work_ctr, 1) + static_cast<int>(gridDim.x);
        w = __shfl_sync(0xffffffffu, w, 0);
      }
      it = producer_load<kT>(a, tail, compact, total, w, lane);
    } while (it.valid == 0);
    return it;
  };
  ProducerItem<kT> nxt = next_item();
  while (nxt.valid > 0) {
    const ProducerItem<kT> cur = nxt;
    // start the next item's counter update before this item's work
    int w_next = 0;
    if (lane == 0) w_next = atomicAdd(work_ctr, 1) + static_cast<int>(gridDim.x);
    const bool stores = cur.split == cur.nsplit - 1 && (a.mode & B2_STORE_KV);
    const int new_idx = stores ? cur.past / kBlock - cur.blk0 : -1;  // block receiving the new token
    // The q/k work of the item: norm + RoPE of its q, k (and the appended k/v
    // rows with a fence, so the TMA read of that tile sees them).
    uint4 packed[kT];
    auto qk_work = [&]() {
      if constexpr (kT > 1) {
        // several new tokens: token t at position past + t; its k/v row is
        // appended by the item whose blocks hold that position
#pragma unroll
        for (int t = 0; t < kT; ++t) {
          if (t >= cur.ntok) break;
          float x[8];
          unpack8(cur.raw[t], x);
          const int pos = cur.past + t;
          const bool rope_ok = pos < a.rope_rows;
          if ((a.mode & B2_ROPE_QK) && !rope_ok && lane == 0 && cur.split == 0 && cur.kvh == 0)
            atomicOr(a.err, B2_DEV_BAD_POSITION);
          const bool rope = grp < 3 && (a.mode & B2_ROPE_QK) && rope_ok;
          norm_rope8(x, j, norm, rope, grp < 2 ? a.gamma_q : a.gamma_k, a.eps,
                     rope ? a.cos + (int64_t)pos * kDim : nullptr, rope ? a.sin + (int64_t)pos * kDim : nullptr);
          packed[t] = pack8(x);
          if (cur.split == 0 && grp < 2 && a.q_out)
            *reinterpret_cast<uint4 *>(a.q_out + (((int64_t)cur.b * a.tokens + t) * kHq + 2 * cur.kvh + grp) * kDim +
                                       j * 8) = packed[t];
          const int idx = pos / kBlock - cur.blk0;  // the same in every lane
          if ((a.mode & B2_STORE_KV) && idx >= 0 && idx < cur.n) {
            const int nb = idx < 32 ? __shfl_sync(0xffffffffu, cur.my_blk, idx)
                                    : __ldg(a.block_tables + (int64_t)cur.b * a.max_blocks + cur.blk0 + idx);
            if (nb < 0 || nb >= a.num_blocks) {
              if (lane == 0) atomicOr(a.err, B2_DEV_BAD_BLOCK);
            } else if (grp >= 2) {
              uint16_t *pool = grp == 2 ? a.k_pool : a.v_pool;
              *reinterpret_cast<uint4 *>(
                  pool + (((int64_t)nb * kHkv + cur.kvh) * kBlock + pos % kBlock) * kDim + j * 8) = packed[t];
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
          }
        }
        return;
      }
      uint4 &packed0 = packed[0];
      float x[8];
      unpack8(cur.raw[0], x);
      const bool rope_ok = cur.past < a.rope_rows;
      if ((a.mode & B2_ROPE_QK) && !rope_ok && lane == 0 && cur.split == 0 && cur.kvh == 0)
        atomicOr(a.err, B2_DEV_BAD_POSITION);
      const bool rope = grp < 3 && (a.mode & B2_ROPE_QK) && rope_ok;
      norm_rope8(x, j, norm, rope, grp < 2 ? a.gamma_q : a.gamma_k, a.eps,
                 rope ? a.cos + (int64_t)cur.past * kDim : nullptr,
                 rope ? a.sin + (int64_t)cur.past * kDim : nullptr);
      packed0 = pack8(x);
      if (cur.split == 0 && grp < 2 && a.q_out)
        *reinterpret_cast<uint4 *>(a.q_out + ((int64_t)cur.b * kHq + 2 * cur.kvh + grp) * kDim + j * 8) = packed0;
      if (stores) {
        // The new token's row lies in this item's last block: write it, then
        // fence so the TMA (async proxy) read of that tile sees the store.
        const int idx = new_idx;  // < n <= 64, the same in every lane
        const int nb = idx < 32 ? __shfl_sync(0xffffffffu, cur.my_blk, idx)
                                : __ldg(a.block_tables + (int64_t)cur.b * a.max_blocks + cur.blk0 + idx);
        if (nb < 0 || nb >= a.num_blocks) {
          if (lane == 0) atomicOr(a.err, B2_DEV_BAD_BLOCK);
        } else if (grp >= 2) {
          uint16_t *pool = grp == 2 ? a.k_pool : a.v_pool;
          *reinterpret_cast<uint4 *>(
              pool + (((int64_t)nb * kHkv + cur.kvh) * kBlock + cur.past % kBlock) * kDim + j * 8) = packed0;
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
      }
    };
    // The item's blocks go out in order, block jj into stage `issued`: wait
    // (bounded) for the stage to be free, write its meta, copy K and V.
    int blk_hi = 0;  // block table entry blk0 + 32 + lane, read at jj == 32
    auto stage_free = [&](int s, uint32_t ph) -> bool {
      int wait_ok = 1;
      if (issued >= kStages && lane == 0) wait_ok = mbar_wait(smem_u32(&tail->empty[s]), ph ^ 1, a.wait_ns);
      wait_ok = __shfl_sync(0xffffffffu, wait_ok, 0);
      if (!wait_ok && lane == 0) atomicOr(a.err, B2_DEV_TIMEOUT);
      return wait_ok != 0;
    };
    auto write_meta = [&](int jj, int s) -> int {
      if (jj == 32)
        blk_hi = lane + 32 < cur.n ? __ldg(a.block_tables + (int64_t)cur.b * a.max_blocks + cur.blk0 + 32 + lane) : 0;
      int blk = __shfl_sync(0xffffffffu, jj < 32 ? cur.my_blk : blk_hi, jj & 31);
      StageMetaT<kT> &m = tail->meta[s];
      if (lane == 0) {
        if constexpr (kT > 1) m.ntok = cur.ntok;
        if (blk < 0 || blk >= a.num_blocks) {
          atomicOr(a.err, B2_DEV_BAD_BLOCK);
          blk = 0;  // read a valid tile instead; the result is flagged as bad
        }
        m.b = cur.b;
        m.kvh = cur.kvh;
        m.split = cur.split;
        m.rows = cur.seq_len - (cur.blk0 + jj) * kBlock;
        m.nsplit = cur.nsplit;
        m.flags = (jj == 0 ? kFlagFirst : 0) | (jj == cur.n - 1 ? kFlagLast : 0) |
                  (cur.nsplit == 1 && a.direct_out ? kFlagFinal : 0);
      }
      return (blk * kHkv + cur.kvh) * kBlock;  // the tile's first row in the pool tensor map
    };
    // The first block.  While the ring fills (the start of the launch: the
    // stage is certainly free) its copies go out before the q/k work and the
    // stage's arrival waits until q is in its meta; later the q/k work runs
    // first, overlapping the wait for a free stage, as the copies could not
    // start earlier anyway.  A first block that receives the new token is
    // copied after the store and its fence in either case.
    const bool early = issued < kStages;
    // (several tokens: some token's position lies in the item's first block)
    const bool first_later = kT == 1 ? new_idx == 0
                                     : (a.mode & B2_STORE_KV) && cur.past / kBlock <= cur.blk0 &&
                                           cur.blk0 <= (cur.past + cur.ntok - 1) / kBlock;
    {
      const int s = issued % kStages;
      const uint32_t full = smem_u32(&tail->full[s]);
      uint8_t *dst = tiles + s * kStageBytes;
      int row = 0;
      if (early) {
        row = write_meta(0, s);
        if (lane == 0) {
          mbar_expect_tx_only(full, kStageBytes);
          if (!first_later) {
            tma_load_2d(smem_u32(dst), tm_k, 0, row, full, policy);
            tma_load_2d(smem_u32(dst + kTileBytes), tm_v, 0, row, full, policy);
          }
        }
      }
      qk_work();
      if (!early) {
        if (!stage_free(s, (issued / kStages) & 1)) {
          ok = false;
          break;
        }
        row = write_meta(0, s);
      }
      if (grp < 2) {
        if constexpr (kT == 1) {
          *reinterpret_cast<uint4 *>(tail->meta[s].q + grp * kDim + j * 8) = packed[0];
        } else {
#pragma unroll
          for (int t = 0; t < kT; ++t)
            if (t < cur.ntok) *reinterpret_cast<uint4 *>(tail->meta[s].q + (2 * t + grp) * kDim + j * 8) = packed[t];
        }
      }
      __syncwarp();
      if (lane == 0) {
        if (!early) mbar_expect_tx(full, kStageBytes);  // arrival + expected bytes
        if (!early || first_later) {
          tma_load_2d(smem_u32(dst), tm_k, 0, row, full, policy);
          tma_load_2d(smem_u32(dst + kTileBytes), tm_v, 0, row, full, policy);
        }
        if (early) mbar_arrive(full);  // q and the meta are in place (release)
      }
      ++issued;
      // the first copy of this item is queued: load the next item now
      w_next = __shfl_sync(0xffffffffu, w_next, 0);
      nxt = producer_load<kT>(a, tail, compact, total, w_next, lane);
    }
    for (int jj = 1; jj < cur.n; ++jj, ++issued) {
      const int s = issued % kStages;
      if (!stage_free(s, (issued / kStages) & 1)) {
        ok = false;
        break;
      }
      const int row = write_meta(jj, s);
      __syncwarp();
      if (lane == 0) {
        const uint32_t full = smem_u32(&tail->full[s]);
        uint8_t *dst = tiles + s * kStageBytes;
        mbar_expect_tx(full, kStageBytes);
        tma_load_2d(smem_u32(dst), tm_k, 0, row, full, policy);
        tma_load_2d(smem_u32(dst + kTileBytes), tm_v, 0, row, full, policy);
      }
    }
    if (!ok) break;
    if (nxt.valid == 0) nxt = next_item();
  }
  if (lane != 0) return;
  int marker = -1;  // stage holding the end-of-work marker
  if (ok) {
    // end-of-work marker: a plain arrival completes the stage's phase
    const int s = issued % kStages;
    const uint32_t ph = (issued / kStages) & 1;
    if (issued < kStages || mbar_wait(smem_u32(&tail->empty[s]), ph ^ 1, a.wait_ns)) {
      tail->meta[s].flags = kFlagEnd;
      mbar_arrive(smem_u32(&tail->full[s]));
      marker = s;
    } else {
      atomicOr(a.err, B2_DEV_TIMEOUT);
    }
  }
  // Wait (bounded) for the copies this CTA issued before leaving.  Normally
  // the consumers have waited for all of them already; a consumer that gave
  // up on a wait may not have.  The marker's stage needs no wait: its last
  // copy was released by the consumers before the marker was placed (the
  // empty wait above), and a parity wait on it would name the wrong phase.
  for (int s = 0; s < kStages && s < issued; ++s) {
    if (s == marker) continue;
    const int last = s + kStages * ((issued - 1 - s) / kStages);
    if (!mbar_wait(smem_u32(&tail->full[s]), (last / kStages) & 1, kDrainLimitNs))
      atomicOr(a.err, B2_DEV_TIMEOUT);
  }
}

// ---- warp-level tensor-core helpers (mma.sync m16n8k16 bf16 -> fp32)

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float c[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) { return pack_bf16x2_rn(lo, hi); }

// Zero the bf16 halves of a fragment register whose token index is >= valid.
__device__ __forceinline__ uint32_t mask_pair(uint32_t v, int tok, int valid) {
  const uint32_t lo = tok < valid ? 0x0000ffffu : 0u;
  const uint32_t hi = tok + 1 < valid ? 0xffff0000u : 0u;
  return v & (lo | hi);
}

// End of an item: merge the 4 warps' states (max and sum per head, output in
// the accumulator layout below).  A whole-sequence item writes the context;
// otherwise the partial state goes to part_ml/part_o for the combine kernel
// that follows.  red[] is double-buffered by epilogue parity, so a single
// barrier separates its writes from its reads and the next epilogue cannot
// overwrite it early.
template <int kT>
__device__ __forceinline__ void step_epilogue(const StepArgs &a, StepTailT<kT> *tail, int warp, int lane, int b,
                                              int kvh, int split, bool final_item, int ntok, float m0, float m1,
                                              float l0, float l1, const float o[4][4], uint32_t &ephase,
                                              int rbuf) {
  float(*red)[2 * kT][2 + kDim] = tail->red[rbuf];
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const int g = lane >> 2, t = lane & 3;
  if constexpr (kT > 1) {
    // lane (g, t) holds token t's state (heads 0, 1) for rows g and g + 8
    if (t < ntok) {
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        red[warp][2 * t][2 + 16 * mt + g] = o[mt][0];
        red[warp][2 * t + 1][2 + 16 * mt + g] = o[mt][1];
        red[warp][2 * t][2 + 16 * mt + g + 8] = o[mt][2];
        red[warp][2 * t + 1][2 + 16 * mt + g + 8] = o[mt][3];
      }
      if (g == 0) {
        red[warp][2 * t][0] = m0;
        red[warp][2 * t][1] = l0;
        red[warp][2 * t + 1][0] = m1;
        red[warp][2 * t + 1][1] = l1;
      }
    }
    consumers_sync(tail, lane, ephase, a.err, a.wait_ns);
    // (token, head) column c = 2 token + head, dim d: merge the 4 warps
    for (int i = threadIdx.x; i < 2 * ntok * kDim; i += kConsumerWarps * 32) {
      const int c = i >> 6, d = i & 63;
      const int tok = c >> 1, h = c & 1;
      float M = -1.0e30f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red[w][c][0]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float sc = ex2(red[w][c][0] - M);
        L = fmaf(red[w][c][1], sc, L);
        O = fmaf(red[w][c][2 + d], sc, O);
      }
      const int64_t row = (int64_t)b * a.tokens + tok;
      if (final_item) {
        a.out[(row * kHq + 2 * kvh + h) * kDim + d] = static_cast<uint16_t>(bf16_bits(O / L));
      } else {
        const int64_t idx = (row * a.num_splits + split) * kHq + 2 * kvh + h;
        a.part_o[idx * kDim + d] = O;
        if (d == 0) {
          a.part_ml[idx * 2] = M;
          a.part_ml[idx * 2 + 1] = L;
        }
      }
    }
    return;
  }
  if (t == 0) {
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      red[warp][0][2 + 16 * mt + g] = o[mt][0];
      red[warp][1][2 + 16 * mt + g] = o[mt][1];
      red[warp][0][2 + 16 * mt + g + 8] = o[mt][2];
      red[warp][1][2 + 16 * mt + g + 8] = o[mt][3];
    }
  }
  if (lane == 0) {
    red[warp][0][0] = m0;
    red[warp][0][1] = l0;
    red[warp][1][0] = m1;
    red[warp][1][1] = l1;
  }
  consumers_sync(tail, lane, ephase, a.err, a.wait_ns);
  const int tid = threadIdx.x;  // 0..127
  const int h = tid >> 6, d = tid & 63;
  float M = -1.0e30f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, red[w][h][0]);
  float L = 0.f, O = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) {
    const float sc = ex2(red[w][h][0] - M);
    L = fmaf(red[w][h][1], sc, L);
    O = fmaf(red[w][h][2 + d], sc, O);
  }
  if (final_item) {
    a.out[((int64_t)b * kHq + 2 * kvh + h) * kDim + d] = static_cast<uint16_t>(bf16_bits(O / L));
    return;
  }
  const int64_t idx = ((int64_t)b * a.num_splits + split) * kHq + 2 * kvh + h;
  a.part_o[idx * kDim + d] = O;
  if (d == 0) {
    a.part_ml[idx * 2] = M;
    a.part_ml[idx * 2 + 1] = L;
  }
}

// Hand an item (or, with b < 0, the end of the work) to the merger warp.
// Every consumer thread arrives (release) after its own stores of the
// partial state, so the merger sees all of them when the phase completes.
template <class Tail>
__device__ __forceinline__ void publish(const StepArgs &a, Tail *tail, int lane, uint32_t &pubs, int b,
                                        int kvh, int split, int nsplit) {
  const int slot = pubs % kPubSlots;
  if (pubs >= kPubSlots && !mbar_wait(smem_u32(&tail->pfree[slot]), ((pubs / kPubSlots) - 1) & 1, a.wait_ns)) {
    if (lane == 0) atomicOr(a.err, B2_DEV_TIMEOUT);
  }
  if (threadIdx.x == 0) tail->pubinfo[slot] = make_int4(b, kvh, split, nsplit);
  // all consumer threads must see the slot free before thread 0 overwrites it:
  // the pfree wait above is done by every thread, and thread 0 writes after it
  mbar_arrive(smem_u32(&tail->pub[slot]));
  ++pubs;
}

// Merger warp: for every published item, count its arrival for (sequence,
// kv head); the last split to arrive merges all splits of the sequence (at
// most kMergeInKernelSplits) into the bf16 context, or into the fp32 state
// when the caller asked for states.  The merge keeps every split's loads in
// flight together (it runs at the tail of the launch for the last sequences):
// lane sp loads split sp's (max, sum) of both heads, the warp reduces the
// maximum and the rescaled sums with shuffles, then each lane accumulates its
// two dims of both heads over the splits, loading eight splits per round.
template <int kT>
__device__ __forceinline__ void step_merger(const StepArgs &a, StepTailT<kT> *tail, int lane) {
  for (uint32_t k = 0;; ++k) {
    const int slot = k % kPubSlots;
    if (!mbar_wait(smem_u32(&tail->pub[slot]), (k / kPubSlots) & 1, a.wait_ns)) {
      if (lane == 0) atomicOr(a.err, B2_DEV_TIMEOUT);
      return;
    }
    const int4 info = tail->pubinfo[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&tail->pfree[slot]));
    if (info.x < 0) return;
    const int b = info.x, kvh = info.y, nsplit = info.w;
    int32_t *cnt = a.counters + 2 + b * kHkv + kvh;
    int last = 0;
    if (lane == 0) {
      __threadfence();  // release the consumers' partial-state stores at GPU scope
      last = atomicAdd(cnt, 1) == nsplit - 1;
      if (last) __threadfence();  // acquire the other CTAs' partial states
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    if (!last) continue;
    // One new token: the merge of (sequence b, kv head) as it stood before
    // several tokens were added (kept apart: in the lambda form below the
    // one-token step measured ~3 us slower at C3).
    if constexpr (kT == 1) {
      const int64_t base = (int64_t)b * a.num_splits * kHq + 2 * kvh;  // (b, split 0, head 2kvh)
      // (max, sum) of heads 2kvh and 2kvh+1 of split `lane`: 4 adjacent floats
      float4 ml = make_float4(-1.0e30f, 0.f, -1.0e30f, 0.f);
      if (lane < nsplit) ml = __ldcg(reinterpret_cast<const float4 *>(a.part_ml + (base + (int64_t)lane * kHq) * 2));
      float M0 = ml.x, M1 = ml.z;
  #pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        M0 = fmaxf(M0, __shfl_xor_sync(0xffffffffu, M0, off));
        M1 = fmaxf(M1, __shfl_xor_sync(0xffffffffu, M1, off));
      }
      const float c0 = ex2(ml.x - M0), c1 = ex2(ml.z - M1);  // lanes past nsplit carry l = 0
      float L0 = ml.y * c0, L1 = ml.w * c1;
  #pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        L0 += __shfl_xor_sync(0xffffffffu, L0, off);
        L1 += __shfl_xor_sync(0xffffffffu, L1, off);
      }
      float2 O0 = make_float2(0.f, 0.f), O1 = make_float2(0.f, 0.f);
      for (int s0 = 0; s0 < nsplit; s0 += 8) {
        float2 v0[8], v1[8];
  #pragma unroll
        for (int e = 0; e < 8; ++e) {
          v0[e] = v1[e] = make_float2(0.f, 0.f);
          if (s0 + e < nsplit) {
            const float *po = a.part_o + (base + (int64_t)(s0 + e) * kHq) * kDim + 2 * lane;
            v0[e] = __ldcg(reinterpret_cast<const float2 *>(po));
            v1[e] = __ldcg(reinterpret_cast<const float2 *>(po + kDim));
          }
        }
  #pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float w0 = __shfl_sync(0xffffffffu, c0, (s0 + e) & 31);
          const float w1 = __shfl_sync(0xffffffffu, c1, (s0 + e) & 31);
          O0.x = fmaf(w0, v0[e].x, O0.x);
          O0.y = fmaf(w0, v0[e].y, O0.y);
          O1.x = fmaf(w1, v1[e].x, O1.x);
          O1.y = fmaf(w1, v1[e].y, O1.y);
        }
      }
      const int64_t oi = ((int64_t)b * kHq + 2 * kvh) * kDim + 2 * lane;
      if (a.direct_out) {
        *reinterpret_cast<uint32_t *>(a.out + oi) = bf16_bits(O0.x / L0) | (bf16_bits(O0.y / L0) << 16);
        *reinterpret_cast<uint32_t *>(a.out + oi + kDim) = bf16_bits(O1.x / L1) | (bf16_bits(O1.y / L1) << 16);
      } else {
        *reinterpret_cast<float2 *>(a.state_o + oi) = O0;
        *reinterpret_cast<float2 *>(a.state_o + oi + kDim) = O1;
        if (lane == 0)
          *reinterpret_cast<float4 *>(a.state_ml + ((int64_t)b * kHq + 2 * kvh) * 2) = make_float4(M0, L0, M1, L1);
      }
    } else {
      // merge the splits of (row, kv head): row = the sequence, or with several
      // new tokens (sequence, token) (info.z carries the sequence's new tokens)
      auto merge_row = [&](int64_t row) {
        const int64_t base = row * a.num_splits * kHq + 2 * kvh;  // (row, split 0, head 2kvh)
        // (max, sum) of heads 2kvh and 2kvh+1 of split `lane`: 4 adjacent floats
        float4 ml = make_float4(-1.0e30f, 0.f, -1.0e30f, 0.f);
        if (lane < nsplit) ml = __ldcg(reinterpret_cast<const float4 *>(a.part_ml + (base + (int64_t)lane * kHq) * 2));
        float M0 = ml.x, M1 = ml.z;
    #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          M0 = fmaxf(M0, __shfl_xor_sync(0xffffffffu, M0, off));
          M1 = fmaxf(M1, __shfl_xor_sync(0xffffffffu, M1, off));
        }
        const float c0 = ex2(ml.x - M0), c1 = ex2(ml.z - M1);  // lanes past nsplit carry l = 0
        float L0 = ml.y * c0, L1 = ml.w * c1;
    #pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
          L0 += __shfl_xor_sync(0xffffffffu, L0, off);
          L1 += __shfl_xor_sync(0xffffffffu, L1, off);
        }
        float2 O0 = make_float2(0.f, 0.f), O1 = make_float2(0.f, 0.f);
        for (int s0 = 0; s0 < nsplit; s0 += 8) {
          float2 v0[8], v1[8];
    #pragma unroll
          for (int e = 0; e < 8; ++e) {
            v0[e] = v1[e] = make_float2(0.f, 0.f);
            if (s0 + e < nsplit) {
              const float *po = a.part_o + (base + (int64_t)(s0 + e) * kHq) * kDim + 2 * lane;
              v0[e] = __ldcg(reinterpret_cast<const float2 *>(po));
              v1[e] = __ldcg(reinterpret_cast<const float2 *>(po + kDim));
            }
          }
    #pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float w0 = __shfl_sync(0xffffffffu, c0, (s0 + e) & 31);
            const float w1 = __shfl_sync(0xffffffffu, c1, (s0 + e) & 31);
            O0.x = fmaf(w0, v0[e].x, O0.x);
            O0.y = fmaf(w0, v0[e].y, O0.y);
            O1.x = fmaf(w1, v1[e].x, O1.x);
            O1.y = fmaf(w1, v1[e].y, O1.y);
          }
        }
        const int64_t oi = (row * kHq + 2 * kvh) * kDim + 2 * lane;
        if (a.direct_out) {
          *reinterpret_cast<uint32_t *>(a.out + oi) = bf16_bits(O0.x / L0) | (bf16_bits(O0.y / L0) << 16);
          *reinterpret_cast<uint32_t *>(a.out + oi + kDim) = bf16_bits(O1.x / L1) | (bf16_bits(O1.y / L1) << 16);
        } else {
          *reinterpret_cast<float2 *>(a.state_o + oi) = O0;
          *reinterpret_cast<float2 *>(a.state_o + oi + kDim) = O1;
          if (lane == 0)
            *reinterpret_cast<float4 *>(a.state_ml + (row * kHq + 2 * kvh) * 2) = make_float4(M0, L0, M1, L1);
        }
      };
      for (int tok = 0; tok < info.z; ++tok) merge_row((int64_t)b * a.tokens + tok);
    }
    if (lane == 0) atomicExch(cnt, 0);
  }
}


// Consumer warp w owns token rows [16w, 16w+16) of every 64-token tile.  Both
// products run on the tensor cores with mma.sync m16n8k16 (bf16 in, fp32
// accumulate), operands fetched from the 128-byte-swizzled tiles with
// ldmatrix; the N = 8 side carries the 2 query heads of the GQA pair (6
// columns are zero):
//   S[16 x 8]  = K_rows[16 x 64] . Q^T[64 x 8]             (4 k-steps)
//   O^T[64 x 8] += V_rows^T[64 x 16] . P^T[16 x 8]           (4 m-tiles)
// Online softmax in fp32 (log2 units); P is rounded to bf16 for the second
// product, as the reference's eager path rounds its probabilities.  Lane
// (g, t) = (lane / 4, lane % 4): scores of rows g and g+8 for both heads live
// in lanes with t == 0; the output accumulator o[mt] holds dims 16mt+g and
// 16mt+g+8 (heads 2t, 2t+1: only t == 0 carries real heads).
template <int kT>
__device__ __forceinline__ void step_consumer(const StepArgs &a, StepTailT<kT> *tail, const uint8_t *tiles, int warp,
                                              int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int j = lane >> 3;  // ldmatrix sub-matrix this lane addresses
  uint32_t bq[4][2];        // Q^T fragments of the current item
  float m0 = -1.0e30f, m1 = -1.0e30f, l0 = 0.f, l1 = 0.f;
  float o[4][4];
#pragma unroll
  for (int mt = 0; mt < 4; ++mt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[mt][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) bq[ks][0] = bq[ks][1] = 0u;
  uint32_t ephase = 0;  // completed phases of the epilogue barrier
  int epilogues = 0;    // red[] buffer parity
  uint32_t pubs = 0;    // items published to the merger warp
  int ntok = 1;         // new tokens of the current item's sequence (kT > 1)
  // ldmatrix row addresses (without the stage base): rows of this lane's
  // sub-matrix, the 16-byte chunk index is added per k-step / m-tile.
  const int qk_row = 16 * warp + (lane & 7) + 8 * (j & 1);
  const int pv_row = 16 * warp + (lane & 7) + 8 * (j >> 1);
  for (int it = 0;; ++it) {
    const int s = it % kStages;
    const uint32_t ph = (it / kStages) & 1;
    if ((a.mode & B2_TEST_STALL) && it == 0 && warp == 0 && blockIdx.x == 0 &&
        !mbar_wait(smem_u32(&tail->stall), 0, a.wait_ns)) {
      // test mode: this warp waits on a barrier that nothing completes, gives
      // up after the wait limit and leaves like a warp that timed out
      if (lane == 0) atomicOr(a.err, B2_DEV_TIMEOUT);
      break;
    }
    if (!mbar_wait(smem_u32(&tail->full[s]), ph, a.wait_ns)) {
      if (lane == 0) atomicOr(a.err, B2_DEV_TIMEOUT);
      break;
    }
    const StageMetaT<kT> &meta = tail->meta[s];
    const int flags = meta.flags;
    if (flags & kFlagEnd) break;
    const int b = meta.b, kvh = meta.kvh, split = meta.split, meta_nsplit = meta.nsplit;
    const int valid = meta.rows - 16 * warp;  // valid rows of this warp (may be <= 0 or >= 16)
    if (flags & kFlagFirst) {
      // B fragment of Q^T: (k = 2t, 2t+1 | 2t+8, 2t+9 of the k-step, n = g)
      // = q[head g][16ks + ...] for g < 2, zero for the padding columns.
      // With several new tokens column g is (token g / 2, head g % 2), as q
      // is laid out [token][head][64] in the meta.
      if constexpr (kT > 1) ntok = meta.ntok;
      const int ncols = kT == 1 ? 2 : 2 * ntok;
      const uint32_t *q32 = reinterpret_cast<const uint32_t *>(meta.q);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        bq[ks][0] = g < ncols ? q32[(g * kDim + 16 * ks + 2 * t) >> 1] : 0u;
        bq[ks][1] = g < ncols ? q32[(g * kDim + 16 * ks + 2 * t + 8) >> 1] : 0u;
      }
      m0 = m1 = -1.0e30f;
      l0 = l1 = 0.f;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[mt][e] = 0.f;
    }
    const uint32_t kt = smem_u32(tiles + s * kStageBytes);
    const uint32_t vt = kt + kTileBytes;

    // S = K . Q^T
    float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int chunk = 2 * ks + (j >> 1);
      uint32_t a0, a1, a2, a3;
      ldsm_x4(kt + qk_row * 128 + ((chunk ^ (qk_row & 7)) << 4), a0, a1, a2, a3);
      mma_bf16(c, a0, a1, a2, a3, bq[ks][0], bq[ks][1]);
    }
    // online softmax over this warp's 16 rows (rows >= valid masked)
    // (several tokens: lane t holds token t, which sees ntok - 1 - t rows
    // fewer than the last token: causal within the new tokens)
    const bool head_lane = kT == 1 ? t == 0 : t < ntok;
    const int tv = kT == 1 ? valid : valid - (ntok - 1 - t);
    const float s00 = head_lane && g < tv ? c[0] * a.scale_log2 : -INFINITY;      // row g,   head 0
    const float s01 = head_lane && g < tv ? c[1] * a.scale_log2 : -INFINITY;      // row g,   head 1
    const float s10 = head_lane && g + 8 < tv ? c[2] * a.scale_log2 : -INFINITY;  // row g+8, head 0
    const float s11 = head_lane && g + 8 < tv ? c[3] * a.scale_log2 : -INFINITY;  // row g+8, head 1
    float bm0 = fmaxf(s00, s10), bm1 = fmaxf(s01, s11);
    // over the rows (lanes of the same t; with one token the other lanes hold -inf)
#pragma unroll
    for (int off = kT == 1 ? 1 : 4; off < 32; off <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
    }
    const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
    const float a0s = ex2(m0 - mn0), a1s = ex2(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const float p00 = ex2(s00 - mn0), p10 = ex2(s10 - mn0);
    const float p01 = ex2(s01 - mn1), p11 = ex2(s11 - mn1);
    l0 = fmaf(l0, a0s, p00 + p10);
    l1 = fmaf(l1, a1s, p01 + p11);
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      o[mt][0] *= a0s;
      o[mt][1] *= a1s;
      o[mt][2] *= a0s;
      o[mt][3] *= a1s;
    }
    // P^T as the B fragment: (k = tokens 2t, 2t+1 | 2t+8, 2t+9, n = head g)
    const uint32_t pk0 = pack_bf16x2(p00, p01);  // row g:   (head 0, head 1)
    const uint32_t pk1 = pack_bf16x2(p10, p11);  // row g+8
    // (several tokens: column g is (token g / 2, head g % 2), whose rows 2t,
    // 2t + 1 sit in lanes 8t + token and 8t + 4 + token)
    const int ptok = kT == 1 ? 0 : g >> 1;
    const uint32_t v0 = __shfl_sync(0xffffffffu, pk0, 8 * t + ptok);
    const uint32_t v1 = __shfl_sync(0xffffffffu, pk0, 8 * t + 4 + ptok);
    const uint32_t v2 = __shfl_sync(0xffffffffu, pk1, 8 * t + ptok);
    const uint32_t v3 = __shfl_sync(0xffffffffu, pk1, 8 * t + 4 + ptok);
    const uint32_t sel = (kT == 1 ? g == 0 : (g & 1) == 0) ? 0x5410u : 0x7632u;
    const int pcols = kT == 1 ? 2 : 2 * ntok;
    const uint32_t bp0 = g < pcols ? __byte_perm(v0, v1, sel) : 0u;
    const uint32_t bp1 = g < pcols ? __byte_perm(v2, v3, sel) : 0u;
    // O^T += V^T . P^T
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
      const int chunk = 2 * mt + (j & 1);
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vt + pv_row * 128 + ((chunk ^ (pv_row & 7)) << 4), a0, a1, a2, a3);
      if (valid < 16) {  // stale or NaN rows past the end must not meet P = 0
        a0 = mask_pair(a0, 2 * t, valid);
        a1 = mask_pair(a1, 2 * t, valid);
        a2 = mask_pair(a2, 2 * t + 8, valid);
        a3 = mask_pair(a3, 2 * t + 8, valid);
      }
      mma_bf16(o[mt], a0, a1, a2, a3, bp0, bp1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&tail->empty[s]));
    if (flags & kFlagLast) {
      const bool final_item = (flags & kFlagFinal) != 0;
      step_epilogue<kT>(a, tail, warp, lane, b, kvh, split, final_item, ntok, m0, m1, l0, l1, o, ephase,
                        (epilogues++) & 1);
      if (!final_item && a.merge_here) publish(a, tail, lane, pubs, b, kvh, kT == 1 ? split : ntok, meta_nsplit);
    }
  }
  publish(a, tail, lane, pubs, -1, 0, 0, 0);  // end of work for the merger warp
}

template <int kT>
__global__ void __launch_bounds__(kStepThreads, step_ctas_per_sm<kT>())
    decode_step_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const StepArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *tiles = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  StepTailT<kT> *tail = reinterpret_cast<StepTailT<kT> *>(tiles + kStages * kStageBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&tail->full[s]), 1);
      mbar_init(smem_u32(&tail->empty[s]), kConsumerWarps);
    }
    mbar_init(smem_u32(&tail->ebar), kConsumerWarps);
    mbar_init(smem_u32(&tail->stall), 1);
#pragma unroll
    for (int s = 0; s < kPubSlots; ++s) {
      mbar_init(smem_u32(&tail->pub[s]), kConsumerWarps * 32);
      mbar_init(smem_u32(&tail->pfree[s]), 1);
    }
    mbar_fence_init();
  }
  __syncthreads();
  // Launched as a programmatic dependent of the previous kernel on the
  // stream: the set-up above overlaps its tail; wait for its completion (and
  // memory) before touching global memory.  A no-op for an ordinary launch.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // A dependent launched with programmatic serialization may start its own
  // set-up now; it waits for this grid's completion before reading memory.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == kProducerWarp)
    step_producer<kT>(a, tail, tiles, &tm_k, &tm_v, lane);
  else if (warp == kMergerWarp)
    step_merger<kT>(a, tail, lane);
  else
    step_consumer<kT>(a, tail, tiles, warp, lane);
  __syncthreads();
  if (threadIdx.x == 0) {
    // The last CTA to finish resets the work counter for the next launch.
    int32_t *work_ctr = a.counters;
    __threadfence();
    if (atomicAdd(work_ctr + 1, 1) == (int)gridDim.x - 1) {
      atomicExch(work_ctr, 0);
      atomicExch(work_ctr + 1, 0);
    }
  }
}

// ------------------------------------------------------------------ batched-prompt attention (tcgen05)

// A chunk of T new tokens per sequence (a prompt, or the x8p engine's
// 4-token batches, experiments/kernels/x8/x8p_core.cc:137-226) attends to
// the cached tokens and causally to the chunk.  Per (64-token query tile, KV
// head, sequence) one CTA holds a 128-row query tile (64 tokens x the GQA
// pair) and streams the sequence's 64-token K/V blocks:
//   S_j[128 x 64]  = Q[128 x 64] . K_j^T     tcgen05.mma, M=128 N=64 K=64, into TMEM
//   O[128 x 64]   += P_j[128 x 64] . V_j     tcgen05.mma accumulating in TMEM
// Warp roles: warp 4 lane 0 feeds K tiles and warp 6 lane 0 V tiles with TMA
// (two 3-stage rings: a K stage is free again once its S product is done, so
// K copies run two to three blocks ahead), warp 5 lane 0 issues the MMAs,
// warps 0-3 run the online softmax (thread = query row = TMEM lane).  S and
// P are double-buffered in TMEM, so the tensor cores compute S_{j+1} and
// P_j.V_j while the softmax of the next block runs; P_j (bf16 pairs written
// with tcgen05.st) is the A operand of its P.V product straight from TMEM,
// with no shared-memory round trip or proxy fence between softmax and MMA.  The running maximum is re-based lazily: a row's O is rescaled
// (TMEM load, scale, store) only when its block maximum exceeds the one in
// use by more than kPfRebase (log2 units); between re-bases P <= 2^kPfRebase,
// well inside bf16 and fp32 range.

constexpr int kPfStages = 3;
constexpr int kPfThreads = 7 * 32;  // 4 softmax warps + K TMA warp + MMA warp + V TMA warp
constexpr int kPfTmemCols = 256;    // S buffers at columns 0 and 64, O at 128, P buffers at 192 and 224
constexpr float kPfRebase = 8.0f;
// Up to this many sequences, CTAs take the sequences longest first (blocks
// launch in blockIdx order, so the longest runs start in the first wave).
constexpr int kPfSortMax = 128;
constexpr uint32_t kPfIdescS = (1u << 4) | (1u << 7) | (1u << 10) | (8u << 17) | (8u << 24);  // f32 <- bf16, M128 N64, K-major
constexpr uint32_t kPfIdescPV = kPfIdescS | (1u << 16);  // B (V) MN-major

struct __align__(8) PrefillTail {
  uint64_t kfull[kPfStages];   // K tile landed (TMA)
  uint64_t kempty[kPfStages];  // K stage read by its S product (commit)
  uint64_t vfull[kPfStages];   // V tile landed (TMA)
  uint64_t vempty[kPfStages];  // V stage read by its P.V product (commit)
  uint64_t sbar[2];           // S_j computed (commit)
  uint64_t sfree[2];          // S_j read by all 128 softmax threads
  uint64_t pready[2];         // P_j written (and O re-based) by all 128 softmax threads
  uint64_t pfree[2];          // P buffer read by its P.V MMA (commit)
  uint64_t pvbar;             // P_j.V_j accumulated (commit, once per block)
  uint64_t obar;              // every product issued done (one commit after the last)
  uint32_t tmem_base;
  int abort;
};
constexpr int kPfSmem = 1024 + 16384 + kPfStages * kStageBytes + (int)sizeof(PrefillTail);

struct PrefillArgs {
  const uint16_t *q;  // [batch][tokens][16][64] normalised + rotated
  const int32_t *block_tables;
  int max_blocks;
  const int32_t *past_lens;
  const int32_t *chunk_lens;
  int tokens;
  int num_blocks;
  float scale_log2;
  uint16_t *out;  // [batch][tokens][16][64]
  int32_t *err;
  // split-KV (bps > 0): blocks [split * bps, (split + 1) * bps) of each tile,
  // partial states to part_ml [nsplit][batch][tokens][16][2] (max in log2
  // units, sum) and part_o [nsplit][batch][tokens][16][64] (unnormalised)
  int bps, nsplit;
  float *part_ml, *part_o;
  uint64_t wait_ns;  // limit of a wait on another warp
};

// Split-KV prefill: the partial state of (split, sequence b, token row, head)
__device__ __forceinline__ void pf_store_part(const PrefillArgs &a, int split, int b, int row, int head, float m,
                                              float l, const float *o) {
  const int64_t r = ((static_cast<int64_t>(split) * gridDim.z / a.nsplit + b) * a.tokens + row) * kHq + head;
  a.part_ml[r * 2] = m;
  a.part_ml[r * 2 + 1] = l;
  float4 *dst = reinterpret_cast<float4 *>(a.part_o + r * kDim);
#pragma unroll
  for (int c = 0; c < kDim; c += 4) dst[c >> 2] = o ? make_float4(o[c], o[c + 1], o[c + 2], o[c + 3])
                                                    : make_float4(0.f, 0.f, 0.f, 0.f);
}

// Shared-memory matrix descriptor for tcgen05.mma: 128-byte swizzle, rows of
// 128 bytes, 8-row groups 1024 bytes apart (SBO); LBO as given (unused for a
// single swizzle atom along the contiguous dimension); version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo_bytes) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(1024u >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// The same with A from tensor memory: M rows = TMEM lanes, K along the
// columns (two bf16 per 32-bit column).
__device__ __forceinline__ void umma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic): one instruction for two lanes'
// worth of FMA / add, halving the softmax's FMA-pipe instructions.
__device__ __forceinline__ void ffma2(float &d0, float &d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void fadd2(float &d0, float &d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane, without waiting
// (several loads in flight; tmem_wait_ld() before using any of them).
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t r[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 16 consecutive fp32 columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float v[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}

// 32 consecutive 32-bit columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t v[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 64 consecutive fp32 columns of this thread's TMEM lane (4 loads, one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float v[64]) {
  uint32_t r[64];
#pragma unroll
  for (int c = 0; c < 64; c += 16) tmem_ld16_nowait(taddr + c, r + c);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__global__ void __launch_bounds__(kPfThreads, 2)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const PrefillArgs a) {
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int nsplit = a.bps > 0 ? a.nsplit : 1;
  const int zb = blockIdx.z / nsplit, split = blockIdx.z % nsplit;  // splits of a sequence are adjacent
  const int nb = gridDim.z / nsplit;
  int b = zb;
  if (nb <= kPfSortMax) {
    // sequence of rank zb by total keys (past + chunk), descending
    __shared__ int keys[kPfSortMax];
    __shared__ int chosen;
    for (int i = threadIdx.x; i < nb; i += blockDim.x)
      keys[i] = a.past_lens[i] + (a.chunk_lens ? a.chunk_lens[i] : a.tokens);
    __syncthreads();
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const int ki = keys[i];
      int rank = 0;
      for (int j2 = 0; j2 < nb; ++j2) rank += (keys[j2] > ki) || (keys[j2] == ki && j2 < i);
      if (rank == zb) chosen = i;
    }
    __syncthreads();
    b = chosen;
  }
  const int past = a.past_lens[b];
  const int T = a.chunk_lens ? a.chunk_lens[b] : a.tokens;
  const int t0 = tile * 64;
  if (t0 >= T) {
    if (a.bps > 0)  // split-KV: empty states for the rows of a tile past the chunk
      for (int i = threadIdx.x; i < 128; i += blockDim.x) {
        const int t = i & 63, hl = i >> 6;
        if (t0 + t < a.tokens) pf_store_part(a, split, b, t0 + t, 2 * kvh + hl, -1.0e30f, 0.f, nullptr);
      }
    return;
  }
  if (past < 0 || T > a.tokens || past + T > a.max_blocks * kBlock) {
    if (threadIdx.x == 0 && tile == 0 && kvh == 0) atomicOr(a.err, B2_DEV_BAD_LENGTH);
    return;
  }
  const int rows_t = min(64, T - t0);
  const int last_key = past + t0 + rows_t - 1;  // the tile's highest query position
  const int nblk_all = last_key / kBlock + 1;
  // this CTA's blocks [j0, j0 + nblk): all of them, or one split's
  const int j0 = a.bps > 0 ? split * a.bps : 0;
  const int nblk = a.bps > 0 ? min(nblk_all - j0, a.bps) : nblk_all;
  if (nblk <= 0) {
    // a split past the tile's last key: empty states for the tile's rows
    for (int i = threadIdx.x; i < 128; i += blockDim.x) {
      const int t = i & 63, hl = i >> 6;
      if (t0 + t < a.tokens) pf_store_part(a, split, b, t0 + t, 2 * kvh + hl, -1.0e30f, 0.f, nullptr);
    }
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  uint8_t *sQ = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *kring = sQ + 16384;                 // kPfStages K tiles of 8 KiB
  uint8_t *vring = kring + kPfStages * kTileBytes;  // kPfStages V tiles of 8 KiB
  PrefillTail *tail = reinterpret_cast<PrefillTail *>(vring + kPfStages * kTileBytes);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kPfStages; ++s) {
      mbar_init(smem_u32(&tail->kfull[s]), 1);
      mbar_init(smem_u32(&tail->kempty[s]), 1);
      mbar_init(smem_u32(&tail->vfull[s]), 1);
      mbar_init(smem_u32(&tail->vempty[s]), 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&tail->sbar[i]), 1);
      mbar_init(smem_u32(&tail->sfree[i]), 128);
      mbar_init(smem_u32(&tail->pready[i]), 128);
      mbar_init(smem_u32(&tail->pfree[i]), 1);
    }
    mbar_init(smem_u32(&tail->pvbar), 1);
    mbar_init(smem_u32(&tail->obar), 1);
    tail->abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tail->tmem_base)),
                 "n"(kPfTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  // query tile: row r = (head of the pair) * 64 + token, 128 bytes, swizzled
  if (tid < 128) {
    const int hl = tid >> 6, t = tid & 63;
    const uint4 *src = reinterpret_cast<const uint4 *>(
        a.q + (((int64_t)b * a.tokens + t0 + t) * kHq + 2 * kvh + hl) * kDim);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 v = t < rows_t ? src[c] : make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4 *>(sQ + tid * 128 + ((c ^ (tid & 7)) << 4)) = v;
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = tail->tmem_base;

  if (warp == 4 || warp == 6) {
    // ---------------- TMA producers: warp 4 the K tiles, warp 6 the V tiles
    if (lane == 0) {
      const bool is_k = warp == 4;
      const CUtensorMap *map = is_k ? &tm_k : &tm_v;
      uint64_t *fullb = is_k ? tail->kfull : tail->vfull;
      uint64_t *emptyb = is_k ? tail->kempty : tail->vempty;
      uint8_t *ringb = is_k ? kring : vring;
      const uint64_t policy = evict_first_policy();
      const int32_t *tbl = a.block_tables + (int64_t)b * a.max_blocks;
      int issued = 0;
      for (int j = 0; j < nblk; ++j) {
        const int s = j % kPfStages;
        const uint32_t ph = (j / kPfStages) & 1;
        if (j >= kPfStages && !mbar_wait(smem_u32(&emptyb[s]), ph ^ 1, a.wait_ns)) {
          atomicOr(a.err, B2_DEV_TIMEOUT);
          tail->abort = 1;
          break;
        }
        if (tail->abort) break;
        int blk = tbl[j0 + j];
        if (blk < 0 || blk >= a.num_blocks) {
          if (is_k) atomicOr(a.err, B2_DEV_BAD_BLOCK);
          blk = 0;
        }
        const int row = (blk * kHkv + kvh) * kBlock;
        const uint32_t full = smem_u32(&fullb[s]);
        mbar_expect_tx(full, kTileBytes);
        tma_load_2d(smem_u32(ringb + s * kTileBytes), map, 0, row, full, policy);
        issued = j + 1;
      }
      // wait (bounded) until every issued copy has landed before leaving
      for (int s = 0; s < kPfStages && s < issued; ++s) {
        const int last = s + kPfStages * ((issued - 1 - s) / kPfStages);
        if (!mbar_wait(smem_u32(&fullb[s]), (last / kPfStages) & 1, kDrainLimitNs))
          atomicOr(a.err, B2_DEV_TIMEOUT);
      }
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer: S_0, S_1, then per block P_j.V_j and S_{j+2}
    if (lane == 0) {
      auto issue_s = [&](int j) -> bool {
        const int s = j % kPfStages;
        if (!mbar_wait(smem_u32(&tail->kfull[s]), (j / kPfStages) & 1, a.wait_ns)) return false;
        if (j >= 2 && !mbar_wait(smem_u32(&tail->sfree[j & 1]), ((j >> 1) - 1) & 1, a.wait_ns)) return false;
        tmem_fence_after();
        const uint32_t kt = smem_u32(kring + s * kTileBytes);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_f16(tmem + 64 * (j & 1), umma_desc(smem_u32(sQ) + 32 * ks, 16), umma_desc(kt + 32 * ks, 16),
                   kPfIdescS, ks > 0);
        umma_commit(smem_u32(&tail->sbar[j & 1]));
        umma_commit(smem_u32(&tail->kempty[s]));
        return true;
      };
      bool ok = issue_s(0) && (nblk < 2 || issue_s(1));
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % kPfStages;
        if (!mbar_wait(smem_u32(&tail->pready[j & 1]), (j >> 1) & 1, a.wait_ns) || tail->abort ||
            !mbar_wait(smem_u32(&tail->vfull[s]), (j / kPfStages) & 1, a.wait_ns)) {
          ok = false;
          break;
        }
        tmem_fence_after();
        const uint32_t vt = smem_u32(vring + s * kTileBytes);
        const uint32_t pt = tmem + 192 + 32 * (j & 1);  // P_j: 16 keys per K step = 8 columns
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_f16_ta(tmem + 128, pt + 8 * ks, umma_desc(vt + 2048 * ks, 0), kPfIdescPV,
                      (j > 0 || ks > 0) ? 1u : 0u);
        umma_commit(smem_u32(&tail->pvbar));
        umma_commit(smem_u32(&tail->pfree[j & 1]));
        umma_commit(smem_u32(&tail->vempty[s]));
        if (j + 2 < nblk) ok = issue_s(j + 2);
      }
      if (!ok) {
        if (!tail->abort) atomicOr(a.err, B2_DEV_TIMEOUT);
        tail->abort = 1;
      }
      // One commit after the last product tracks every product issued: its
      // single phase tells this warp (before the CTA frees its TMEM) and the
      // softmax warps (before they read O) that all of them are done.  A parity
      // wait on pvbar could not: it is exact only while pvbar is within one
      // phase of the completion waited for, and here it may lag by two.
      umma_commit(smem_u32(&tail->obar));
      if (!mbar_wait(smem_u32(&tail->obar), 0, kDrainLimitNs)) atomicOr(a.err, B2_DEV_TIMEOUT);
    }
  } else {
    // ---------------- softmax warps: thread = query row = TMEM lane
    const int hl = tid >> 6, t = tid & 63;
    const bool row_ok = t < rows_t;
    const int qpos = past + t0 + t;
    const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
    float m = -1.0e30f, l = 0.f;  // max in use (log2 units) and running sum
    bool ok = true;
    // Waits decided for the whole warp (the TMEM loads and stores below are
    // warp-collective): false if any lane timed out or the CTA is aborting.
    auto warp_wait = [&](uint32_t bar, uint32_t parity) -> bool {
      const bool got = mbar_wait(bar, parity, a.wait_ns);
      return !__any_sync(0xffffffffu, !got || tail->abort);
    };
    // A warp whose 32 rows are all past the chunk (tiles of fewer than 33
    // tokens) keeps step with the barriers but computes nothing: its P rows
    // only feed O rows that are never stored.
    const bool warp_active = __any_sync(0xffffffffu, row_ok);
    for (int j = 0; j < nblk && !warp_active; ++j) {
      const int s = j % kPfStages;
      if (!warp_wait(smem_u32(&tail->sbar[j & 1]), (j >> 1) & 1)) {
        ok = false;
        break;
      }
      mbar_arrive(smem_u32(&tail->sfree[j & 1]));
      if (j >= 2 && !warp_wait(smem_u32(&tail->pfree[j & 1]), ((j >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      const int key0 = (j0 + j) * kBlock;
      if (key0 + kBlock - 1 > last_key) {
        // this thread's share of zeroing the V rows past the tile (below)
        if (!warp_wait(smem_u32(&tail->vfull[s]), (j / kPfStages) & 1)) {
          ok = false;
          break;
        }
        const int first_bad = last_key - key0 + 1;
        uint8_t *v_gen = vring + s * kTileBytes;
        for (int i = tid; i < (kBlock - first_bad) * 8; i += 128)
          *reinterpret_cast<uint4 *>(v_gen + (first_bad + (i >> 3)) * 128 + ((i & 7) << 4)) = make_uint4(0, 0, 0, 0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      mbar_arrive(smem_u32(&tail->pready[j & 1]));
    }
    for (int j = 0; j < nblk && warp_active; ++j) {
      const int s = j % kPfStages;
      if (!warp_wait(smem_u32(&tail->sbar[j & 1]), (j >> 1) & 1)) {
        ok = false;
        break;
      }
      tmem_fence_after();
      float sc[64];
      tmem_ld64(trow + 64 * (j & 1), sc);
      tmem_fence_before();
      mbar_arrive(smem_u32(&tail->sfree[j & 1]));  // S_j is in registers: its buffer may be reused
      // scores of this row, masked: causal within the chunk, nothing past the
      // tile; max in 8 independent chains
      const int key0 = (j0 + j) * kBlock;
      const int lim = row_ok ? qpos - key0 : -1;  // columns c <= lim are visible
      float bm8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) bm8[e] = -INFINITY;
      // raw scores (the scale is folded into the exponent); the mask only
      // where a row of this warp needs it (the tile's diagonal block, rows
      // past the chunk)
      if (__any_sync(0xffffffffu, lim < kBlock - 1)) {
#pragma unroll
        for (int c = 0; c < 64; ++c) sc[c] = c <= lim ? sc[c] : -INFINITY;
      }
#pragma unroll
      for (int c = 0; c < 64; ++c) bm8[c & 7] = fmaxf(bm8[c & 7], sc[c]);
      const float bm = fmaxf(fmaxf(fmaxf(bm8[0], bm8[1]), fmaxf(bm8[2], bm8[3])),
                             fmaxf(fmaxf(bm8[4], bm8[5]), fmaxf(bm8[6], bm8[7]))) * a.scale_log2;
      // re-base when this block's maximum is well above the one in use
      const bool rebase = bm > m + kPfRebase;
      const float mn = rebase ? bm : m;
      const float alpha = ex2(m - mn);  // 1 when not re-based
      if (__any_sync(0xffffffffu, rebase && j > 0)) {
        // O holds P_0..P_{j-1} . V: wait for the last product, then scale
        // this warp's rows in TMEM (alpha = 1 for rows not re-based)
        if (!warp_wait(smem_u32(&tail->pvbar), (j - 1) & 1)) {
          ok = false;
          break;
        }
        tmem_fence_after();
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
          uint32_t r[16];
          tmem_ld16_nowait(trow + 128 + c, r);
          tmem_wait_ld();
          float o16[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) o16[e] = __uint_as_float(r[e]) * alpha;
          tmem_st16(trow + 128 + c, o16);
        }
        tmem_wait_st();
      }
      m = mn;
      float ps8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) ps8[e] = 0.f;
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        float x0, x1;
        ffma2(x0, x1, sc[c], sc[c + 1], a.scale_log2, a.scale_log2, -mn, -mn);
        sc[c] = ex2(x0);
        sc[c + 1] = ex2(x1);
        const int e = c & 7;
        fadd2(ps8[e], ps8[e + 1], ps8[e], ps8[e + 1], sc[c], sc[c + 1]);
      }
      const float ps = ((ps8[0] + ps8[1]) + (ps8[2] + ps8[3])) + ((ps8[4] + ps8[5]) + (ps8[6] + ps8[7]));
      l = fmaf(l, alpha, ps);
      // P_j into buffer j % 2 once the product that read it (P_{j-2}) is done
      if (j >= 2 && !warp_wait(smem_u32(&tail->pfree[j & 1]), ((j >> 1) - 1) & 1)) {
        ok = false;
        break;
      }
      {
        uint32_t pk[32];  // P_j of this row as bf16 pairs, into TMEM buffer j % 2
#pragma unroll
        for (int c = 0; c < 64; c += 2) pk[c >> 1] = pack_bf16x2_rn(sc[c], sc[c + 1]);
        tmem_st32(trow + 192 + 32 * (j & 1), pk);
        tmem_wait_st();
      }
      if (key0 + kBlock - 1 > last_key) {
        // rows of the last block past every query of the tile may hold stale
        // (even NaN) data: zero them so that P = 0 cannot meet them in P.V
        // (after the stage's copy has landed, so the copy cannot overwrite)
        if (!warp_wait(smem_u32(&tail->vfull[s]), (j / kPfStages) & 1)) {
          ok = false;
          break;
        }
        const int first_bad = last_key - key0 + 1;
        uint8_t *v_gen = vring + s * kTileBytes;
        for (int i = tid; i < (kBlock - first_bad) * 8; i += 128)
          *reinterpret_cast<uint4 *>(v_gen + (first_bad + (i >> 3)) * 128 + ((i & 7) << 4)) = make_uint4(0, 0, 0, 0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before the P.V product reads V
      }
      tmem_fence_before();
      mbar_arrive(smem_u32(&tail->pready[j & 1]));
    }
    if (!ok) {
      if (!tail->abort) atomicOr(a.err, B2_DEV_TIMEOUT);
      tail->abort = 1;
    } else if (warp_wait(smem_u32(&tail->obar), 0)) {
      // O = sum_j P_j . V_j, every product done
      tmem_fence_after();
      float o[64];
      tmem_ld64(trow + 128, o);
      if (a.bps > 0 && !tail->abort) {
        // split-KV: the partial state (rows past the chunk get empty states)
        if (t0 + t < a.tokens)
          pf_store_part(a, split, b, t0 + t, 2 * kvh + hl, row_ok ? m : -1.0e30f, row_ok ? l : 0.f,
                        row_ok ? o : nullptr);
      } else if (row_ok && !tail->abort) {
        const float inv = 1.0f / l;
        uint4 *dst =
            reinterpret_cast<uint4 *>(a.out + (((int64_t)b * a.tokens + t0 + t) * kHq + 2 * kvh + hl) * kDim);
#pragma unroll
        for (int c = 0; c < 64; c += 8) {
          float o8[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) o8[e] = o[c + e] * inv;
          dst[c >> 3] = pack8(o8);
        }
      }
    } else {
      atomicOr(a.err, B2_DEV_TIMEOUT);
      tail->abort = 1;
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 0) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kPfTmemCols));
  }
}

// ------------------------------------------------------------------ host helpers

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {  // initialised once, thread-safe
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

// Pool viewed as a 2-D tensor: 64 bf16 per row, num_blocks*8*64 rows; a box
// is one (block, head) tile of 64 rows, swizzled in 128-byte groups.
int encode_pool_map(CUtensorMap *map, const void *pool, int num_blocks) {
  auto fn = encode_fn();
  if (!fn) return fail(B2_ERR_NOSYM, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kDim),
                              static_cast<cuuint64_t>(num_blocks) * kHkv * kBlock};
  const cuuint64_t strides[1] = {kDim * 2};
  const cuuint32_t box[2] = {kDim, kBlock};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(pool), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B2_ERR_ARG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return B2_OK;
}

// The pool's tensor map, encoded once per (pool, num_blocks) and calling
// thread: a decode loop launches on the same pools every step, and the
// encode is host work on the launch path.  The map describes only the
// address range, so a pool freed and allocated again at the same address and
// size is described by the same map.
int make_pool_map(CUtensorMap *map, const void *pool, int num_blocks) {
  struct Entry {
    const void *pool;
    int num_blocks;
    CUtensorMap map;
  };
  constexpr int kEntries = 8;
  thread_local Entry cache[kEntries] = {};
  thread_local int next = 0;
  for (int i = 0; i < kEntries; ++i)
    if (cache[i].pool == pool && cache[i].num_blocks == num_blocks && pool) {
      *map = cache[i].map;
      return B2_OK;
    }
  const int rc = encode_pool_map(map, pool, num_blocks);
  if (rc == B2_OK) {
    cache[next] = Entry{pool, num_blocks, *map};
    next = (next + 1) % kEntries;
  }
  return rc;
}

// Wait limits of the launches (b2_set_wait_limits), read at every launch.
std::atomic<uint64_t> g_wait_ns{kWaitLimitNs};
std::atomic<uint64_t> g_poll_ns{kXWaitNs};
constexpr int64_t kMaxWaitLimitNs = 60000000000ll;

uint64_t wait_limit() { return g_wait_ns.load(std::memory_order_relaxed); }
uint64_t poll_limit() { return g_poll_ns.load(std::memory_order_relaxed); }

int launch_status(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(B2_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return ok();
}

bool decode_smem_ready() {
  // cudaFuncSetAttribute is per device; remember which devices are set up.
  static std::atomic<bool> done[128];  // per device; several host threads may launch at once
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return false;
  if (!done[dev]) {
    if (cudaFuncSetAttribute(paged_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kDecodeSmem) != cudaSuccess)
      return false;
    done[dev] = true;
  }
  return true;
}

template <int kT>
bool step_smem_ready() {
  static std::atomic<bool> done[128];  // per device; several host threads may launch at once
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return false;
  if (!done[dev]) {
    if (cudaFuncSetAttribute(decode_step_kernel<kT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             step_smem<kT>()) != cudaSuccess)
      return false;
    done[dev] = true;
  }
  return true;
}

int sm_count() {
  static std::atomic<int> count[128];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return 148;
  if (!count[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    count[dev] = n;
  }
  return count[dev];
}

}  // namespace

// ------------------------------------------------------------------ C ABI

int b2_record_error(int code, const char *message) { return fail(code, "%s", message); }
uint64_t b2_wait_limit_ns() { return wait_limit(); }
int b2_clear_error() { return ok(); }

extern "C" int b2_version(void) { return 100; }

extern "C" int b2_set_wait_limits(int64_t wait_ns, int64_t poll_ns) {
  if (wait_ns > kMaxWaitLimitNs || poll_ns > kMaxWaitLimitNs)
    return fail(B2_ERR_ARG, "wait limits must be <= %lld ns", (long long)kMaxWaitLimitNs);
  g_wait_ns.store(wait_ns > 0 ? static_cast<uint64_t>(wait_ns) : kWaitLimitNs);
  g_poll_ns.store(poll_ns > 0 ? static_cast<uint64_t>(poll_ns) : kXWaitNs);
  return ok();
}

extern "C" int b2_get_wait_limits(int64_t *wait_ns, int64_t *poll_ns) {
  if (wait_ns) *wait_ns = static_cast<int64_t>(wait_limit());
  if (poll_ns) *poll_ns = static_cast<int64_t>(poll_limit());
  return ok();
}

extern "C" int b2_last_error(char *buf, int len) {
  const int n = static_cast<int>(strlen(g_err));
  if (buf && len > 0) {
    const int m = n < len - 1 ? n : len - 1;
    memcpy(buf, g_err, m);
    buf[m] = 0;
  }
  return n;
}

extern "C" int b2_append_rope(const uint16_t *qkv, int64_t row_stride, const uint16_t *gamma_q,
                              const uint16_t *gamma_k, float eps, const uint16_t *rope_cos,
                              const uint16_t *rope_sin, int32_t rope_rows, const int32_t *past_lens,
                              const int32_t *block_tables, int32_t max_blocks_per_seq,
                              uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks, uint16_t *q_out,
                              int32_t batch, int32_t mode, int32_t *dev_err, void *stream) {
  if (batch < 0) return fail(B2_ERR_ARG, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return ok();
  if (!qkv || !past_lens || !dev_err) return fail(B2_ERR_ARG, "qkv, past_lens and dev_err are required");
  if (mode & ~(B2_NORM_QK | B2_ROPE_QK | B2_STORE_KV)) return fail(B2_ERR_ARG, "unknown mode bits 0x%x", mode);
  if (row_stride < kQkvWidth || row_stride % 8 != 0)
    return fail(B2_ERR_ARG, "row_stride must be >= %d and a multiple of 8 (got %lld)", kQkvWidth,
                (long long)row_stride);
  if (!aligned16(qkv) || (q_out && !aligned16(q_out)))
    return fail(B2_ERR_ARG, "qkv and q_out must be 16-byte aligned");
  if ((mode & B2_NORM_QK) && (!gamma_q || !gamma_k || !aligned16(gamma_q) || !aligned16(gamma_k)))
    return fail(B2_ERR_ARG, "B2_NORM_QK needs 16-byte aligned gamma_q and gamma_k");
  if ((mode & B2_ROPE_QK) &&
      (!rope_cos || !rope_sin || rope_rows <= 0 || !aligned16(rope_cos) || !aligned16(rope_sin)))
    return fail(B2_ERR_ARG, "B2_ROPE_QK needs 16-byte aligned cos/sin tables with rope_rows > 0");
  if (max_blocks_per_seq > kMaxTableWidth) return table_width_error(max_blocks_per_seq);
  if (mode & B2_STORE_KV) {
    if (!block_tables || !k_pool || !v_pool || max_blocks_per_seq <= 0 || num_blocks <= 0)
      return fail(B2_ERR_ARG, "B2_STORE_KV needs block_tables, k_pool, v_pool and positive sizes");
    if (!aligned16(k_pool) || !aligned16(v_pool)) return fail(B2_ERR_ARG, "pools must be 16-byte aligned");
  }
  AppendArgs a{qkv, row_stride, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_lens,
               block_tables, max_blocks_per_seq > 0 ? max_blocks_per_seq : 1, k_pool, v_pool,
               num_blocks, q_out, mode, dev_err, 1, nullptr};
  append_rope_kernel<<<batch, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("append_rope_kernel");
}

extern "C" int b2_decode_attn(const uint16_t *q, const uint16_t *k_pool, const uint16_t *v_pool,
                              int32_t num_blocks, const int32_t *block_tables,
                              int32_t max_blocks_per_seq, const int32_t *seq_lens, int32_t batch,
                              int32_t blocks_per_split, int32_t num_splits, float scale,
                              float *part_ml, float *part_o, int32_t *dev_err, void *stream) {
  if (batch < 0) return fail(B2_ERR_ARG, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return ok();
  if (!q || !k_pool || !v_pool || !block_tables || !seq_lens || !part_ml || !part_o || !dev_err)
    return fail(B2_ERR_ARG, "null pointer argument");
  if (num_blocks <= 0 || static_cast<int64_t>(num_blocks) * kHkv * kBlock >= (int64_t(1) << 31))
    return fail(B2_ERR_ARG, "num_blocks must be in [1, 2^22) (got %d)", num_blocks);
  if (max_blocks_per_seq <= 0 || blocks_per_split <= 0)
    return fail(B2_ERR_ARG, "max_blocks_per_seq and blocks_per_split must be positive");
  if (max_blocks_per_seq > kMaxTableWidth) return table_width_error(max_blocks_per_seq);
  if (blocks_per_split > kMaxTableWidth)
    return fail(B2_ERR_ARG, "blocks_per_split must be <= %d (got %d)", kMaxTableWidth, blocks_per_split);
  if (static_cast<int64_t>(num_splits) * blocks_per_split < max_blocks_per_seq)
    return fail(B2_ERR_ARG, "num_splits * blocks_per_split (%d * %d) < max_blocks_per_seq (%d)",
                num_splits, blocks_per_split, max_blocks_per_seq);
  if (num_splits > 65535 || batch > 65535) return fail(B2_ERR_ARG, "num_splits and batch must be <= 65535");
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool))
    return fail(B2_ERR_ARG, "q and the pools must be 16-byte aligned");
  if (!(scale > 0.f)) return fail(B2_ERR_ARG, "scale must be positive");
  CUtensorMap mk, mv;
  int rc = make_pool_map(&mk, k_pool, num_blocks);
  if (rc) return rc;
  rc = make_pool_map(&mv, v_pool, num_blocks);
  if (rc) return rc;
  if (!decode_smem_ready()) return fail(B2_ERR_CUDA, "cannot set the decode kernel's shared memory size");
  DecodeArgs a{q, block_tables, max_blocks_per_seq, seq_lens, num_blocks, blocks_per_split, num_splits,
               scale * 1.4426950408889634f, part_ml, part_o, dev_err, wait_limit()};
  const dim3 grid(num_splits, kHkv, batch);
  paged_decode_kernel<<<grid, kDecodeThreads, kDecodeSmem, static_cast<cudaStream_t>(stream)>>>(mk, mv, a);
  return launch_status("paged_decode_kernel");
}

extern "C" int b2_combine(const float *part_ml, const float *part_o, int32_t num_parts,
                          const int32_t *seq_lens, int32_t blocks_per_split, int32_t batch,
                          uint16_t *out, float *state_ml, float *state_o, void *stream) {
  if (batch < 0) return fail(B2_ERR_ARG, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return ok();
  if (!part_ml || !part_o || num_parts <= 0) return fail(B2_ERR_ARG, "partial states and num_parts > 0 required");
  if (seq_lens && blocks_per_split <= 0) return fail(B2_ERR_ARG, "blocks_per_split must be positive");
  if (static_cast<int64_t>(num_parts) * (seq_lens ? blocks_per_split : 1) * kBlock > 0x7fffffff)
    return fail(B2_ERR_ARG, "num_parts x blocks_per_split x 64 must fit an int32 token count");
  if (!out && !state_o) return fail(B2_ERR_ARG, "one of out or state_o is required");
  if ((state_o == nullptr) != (state_ml == nullptr)) return fail(B2_ERR_ARG, "state_ml and state_o go together");
  CombineArgs a{part_ml, part_o, num_parts, seq_lens, blocks_per_split, out, state_ml, state_o, 0, 0,
                num_parts * (seq_lens ? blocks_per_split : 1) * kBlock, 0, 0, 0, 0, combine_groups(num_parts)};
  combine_kernel<<<dim3(batch, kHq), a.groups * kDim, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("combine_kernel");
}

extern "C" int b2_decode_step_counters(int32_t batch) { return batch < 0 ? 0 : 2 + batch * kHkv; }

namespace {

// The decode step; with `x` (a multi-GPU exchange), the splits are always
// merged by the combine kernel, which exchanges the merged state with the
// other ranks and writes the world's context into out.
int decode_step_impl(const uint16_t *qkv, int64_t row_stride, const uint16_t *gamma_q, const uint16_t *gamma_k,
                     float eps, const uint16_t *rope_cos, const uint16_t *rope_sin, int32_t rope_rows,
                     const int32_t *past_lens, const int32_t *seq_lens, const int32_t *block_tables,
                     int32_t max_blocks_per_seq, uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks,
                     int32_t batch, int32_t blocks_per_split, float scale, int32_t mode, uint16_t *out,
                     uint16_t *q_out, float *state_ml, float *state_o, float *part_ml, float *part_o,
                     int32_t *counters, int32_t max_ctas, int32_t *dev_err, void *stream, const XchgArgs *x,
                     int32_t tokens = 1, const int32_t *chunk_lens = nullptr) {
  if (batch < 0) return fail(B2_ERR_ARG, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return ok();
  if (tokens < 1 || tokens > kMaxStepTokens) return fail(B2_ERR_ARG, "tokens must be in [1, %d]", kMaxStepTokens);
  if (tokens > 1 && (x || !out || state_o || state_ml || seq_lens))
    return fail(B2_ERR_ARG, "several new tokens: out is required; no states, seq_lens or exchange");
  if (tokens > 1 && (int64_t)batch * tokens > 0x7fffffff) return fail(B2_ERR_ARG, "batch * tokens too large");
  if (!qkv || !past_lens || !block_tables || !k_pool || !v_pool || !part_ml || !part_o || !counters || !dev_err)
    return fail(B2_ERR_ARG, "null pointer argument");
  if (x && (!out || state_o || state_ml)) return fail(B2_ERR_ARG, "an exchange writes out and no state");
  if (!out && !state_o) return fail(B2_ERR_ARG, "one of out or state_o is required");
  if ((state_o == nullptr) != (state_ml == nullptr)) return fail(B2_ERR_ARG, "state_ml and state_o go together");
  if (mode & ~(B2_NORM_QK | B2_ROPE_QK | B2_STORE_KV | B2_TEST_STALL))
    return fail(B2_ERR_ARG, "unknown mode bits 0x%x", mode);
  if (row_stride < kQkvWidth || row_stride % 8 != 0)
    return fail(B2_ERR_ARG, "row_stride must be >= %d and a multiple of 8", kQkvWidth);
  if (!aligned16(qkv) || (out && !aligned16(out)) || (q_out && !aligned16(q_out)) || !aligned16(k_pool) ||
      !aligned16(v_pool))
    return fail(B2_ERR_ARG, "qkv, out, q_out and the pools must be 16-byte aligned");
  if ((mode & B2_NORM_QK) && (!gamma_q || !gamma_k || !aligned16(gamma_q) || !aligned16(gamma_k)))
    return fail(B2_ERR_ARG, "B2_NORM_QK needs 16-byte aligned gamma_q and gamma_k");
  if ((mode & B2_ROPE_QK) &&
      (!rope_cos || !rope_sin || rope_rows <= 0 || !aligned16(rope_cos) || !aligned16(rope_sin)))
    return fail(B2_ERR_ARG, "B2_ROPE_QK needs 16-byte aligned cos/sin tables with rope_rows > 0");
  if (num_blocks <= 0 || static_cast<int64_t>(num_blocks) * kHkv * kBlock >= (int64_t(1) << 31))
    return fail(B2_ERR_ARG, "num_blocks must be in [1, 2^22) (got %d)", num_blocks);
  if (max_blocks_per_seq <= 0) return fail(B2_ERR_ARG, "max_blocks_per_seq must be positive");
  if (max_blocks_per_seq > kMaxTableWidth) return table_width_error(max_blocks_per_seq);
  if (blocks_per_split < 1 || blocks_per_split > kStepMaxBlocksPerSplit)
    return fail(B2_ERR_ARG, "blocks_per_split must be in [1, %d] (got %d)", kStepMaxBlocksPerSplit, blocks_per_split);
  if (!(scale > 0.f)) return fail(B2_ERR_ARG, "scale must be positive");
  if (!aligned16(part_ml) || !aligned16(part_o) || (state_ml && !aligned16(state_ml)) ||
      (state_o && !aligned16(state_o)))
    return fail(B2_ERR_ARG, "part_ml, part_o, state_ml and state_o must be 16-byte aligned");
  const int64_t splits = (static_cast<int64_t>(max_blocks_per_seq) + blocks_per_split - 1) / blocks_per_split;
  const int64_t total = splits * batch * kHkv;
  if (total >= (int64_t(1) << 31)) return fail(B2_ERR_ARG, "too many work items");
  if (tokens > 1 && splits > kMergeInKernelSplits)
    return fail(B2_ERR_ARG,
                "several new tokens need at most %d splits per sequence: blocks_per_split >= ceil(%d / %d)",
                kMergeInKernelSplits, max_blocks_per_seq, kMergeInKernelSplits);
  CUtensorMap mk, mv;
  int rc = make_pool_map(&mk, k_pool, num_blocks);
  if (rc) return rc;
  rc = make_pool_map(&mv, v_pool, num_blocks);
  if (rc) return rc;
  if (!(tokens == 1 ? step_smem_ready<1>() : step_smem_ready<kMaxStepTokens>()))
    return fail(B2_ERR_CUDA, "cannot set the decode-step kernel's shared memory size");
  const int direct_out = state_o == nullptr && !x;
  // One warp merges a (sequence, kv head)'s splits serially: right for a
  // handful of splits; long single sequences with many splits are merged by
  // the parallel combine kernel instead (always, with an exchange).
  const int merge_here = splits <= kMergeInKernelSplits && !x;
  StepArgs a{qkv, row_stride, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_lens, seq_lens,
             block_tables, max_blocks_per_seq, k_pool, v_pool, num_blocks, batch, blocks_per_split,
             static_cast<int>(splits), static_cast<int>(total), direct_out, merge_here,
             scale * 1.4426950408889634f, mode, x ? nullptr : out, q_out, state_ml, state_o, part_ml, part_o,
             counters, dev_err, wait_limit(), tokens, chunk_lens};
  int64_t ctas = static_cast<int64_t>(sm_count()) *
                 (tokens == 1 ? step_ctas_per_sm<1>() : step_ctas_per_sm<kMaxStepTokens>());
  if (max_ctas > 0 && max_ctas < ctas) ctas = max_ctas;
  if (ctas > total) ctas = total;
  // Equal waves: items are handed out dynamically, so with `waves` rounds the
  // last round should be as full as the others (e.g. 520 items run as 2 x 260
  // rather than 444 + 76; every CTA then streams the same number of blocks).
  const int64_t waves = (total + ctas - 1) / ctas;
  ctas = (total + waves - 1) / waves;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  {
    // programmatic dependent of the previous kernel on the stream (see the
    // griddepcontrol.wait at the top of the kernel)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = tokens == 1 ? step_smem<1>() : step_smem<kMaxStepTokens>();
    cfg.stream = st;
    cfg.attrs = pdl;
    cfg.numAttrs = 1;
    const cudaError_t le = tokens == 1 ? cudaLaunchKernelEx(&cfg, decode_step_kernel<1>, mk, mv, a)
                                       : cudaLaunchKernelEx(&cfg, decode_step_kernel<kMaxStepTokens>, mk, mv, a);
    if (le != cudaSuccess) {
      const cudaError_t e = cudaGetLastError();
      return fail(B2_ERR_CUDA, "decode_step_kernel launch failed: %s", cudaGetErrorString(e));
    }
  }
  rc = launch_status("decode_step_kernel");
  if (rc || merge_here) return rc;
  // Many splits: merge them with the parallel combine kernel, launched as a
  // programmatic dependent so that its launch overlaps the decode tail.
  CombineArgs c{part_ml, part_o, static_cast<int>(splits), seq_lens ? seq_lens : past_lens, blocks_per_split,
                x ? nullptr : out, state_ml, state_o, seq_lens ? 0 : 1, direct_out,
                static_cast<int>(splits) * blocks_per_split * kBlock, 0, 0, 0, 0,
                combine_groups(static_cast<int>(splits))};
  if (x) c.x = *x;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(batch), kHq);
  cfg.blockDim = dim3(c.groups * kDim);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, combine_kernel, c) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    return fail(B2_ERR_CUDA, "combine_kernel launch failed: %s", cudaGetErrorString(e));
  }
  return launch_status("combine_kernel (decode step)");
}

}  // namespace

extern "C" int b2_decode_step(const uint16_t *qkv, int64_t row_stride, const uint16_t *gamma_q,
                              const uint16_t *gamma_k, float eps, const uint16_t *rope_cos,
                              const uint16_t *rope_sin, int32_t rope_rows, const int32_t *past_lens,
                              const int32_t *seq_lens, const int32_t *block_tables, int32_t max_blocks_per_seq,
                              uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks, int32_t batch,
                              int32_t blocks_per_split, float scale, int32_t mode, uint16_t *out,
                              uint16_t *q_out, float *state_ml, float *state_o, float *part_ml, float *part_o,
                              int32_t *counters, int32_t max_ctas, int32_t *dev_err, void *stream) {
  return decode_step_impl(qkv, row_stride, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_lens, seq_lens,
                          block_tables, max_blocks_per_seq, k_pool, v_pool, num_blocks, batch, blocks_per_split,
                          scale, mode, out, q_out, state_ml, state_o, part_ml, part_o, counters, max_ctas, dev_err,
                          stream, nullptr);
}

extern "C" int b2_decode_step_tokens(const uint16_t *qkv, int64_t row_stride, int32_t tokens,
                                     const int32_t *chunk_lens, const uint16_t *gamma_q, const uint16_t *gamma_k,
                                     float eps, const uint16_t *rope_cos, const uint16_t *rope_sin,
                                     int32_t rope_rows, const int32_t *past_lens, const int32_t *block_tables,
                                     int32_t max_blocks_per_seq, uint16_t *k_pool, uint16_t *v_pool,
                                     int32_t num_blocks, int32_t batch, int32_t blocks_per_split, float scale,
                                     int32_t mode, uint16_t *out, uint16_t *q_out, float *part_ml, float *part_o,
                                     int32_t *counters, int32_t max_ctas, int32_t *dev_err, void *stream) {
  if (!out) return fail(B2_ERR_ARG, "out is required");
  return decode_step_impl(qkv, row_stride, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_lens, nullptr,
                          block_tables, max_blocks_per_seq, k_pool, v_pool, num_blocks, batch, blocks_per_split,
                          scale, mode, out, q_out, nullptr, nullptr, part_ml, part_o, counters, max_ctas, dev_err,
                          stream, nullptr, tokens, tokens > 1 ? chunk_lens : nullptr);
}

extern "C" int b2_decode_step_exchange(const uint16_t *qkv, int64_t row_stride, const uint16_t *gamma_q,
                                       const uint16_t *gamma_k, float eps, const uint16_t *rope_cos,
                                       const uint16_t *rope_sin, int32_t rope_rows, const int32_t *past_lens,
                                       const int32_t *seq_lens, const int32_t *block_tables,
                                       int32_t max_blocks_per_seq, uint16_t *k_pool, uint16_t *v_pool,
                                       int32_t num_blocks, int32_t batch, int32_t blocks_per_split, float scale,
                                       int32_t mode, uint16_t *out, uint16_t *q_out, float *part_ml, float *part_o,
                                       int32_t *counters, int32_t max_ctas, void *const *areas, int32_t world,
                                       int32_t rank, int32_t *dev_err, void *stream) {
  if (batch > 65535) return fail(B2_ERR_ARG, "batch must be <= 65535");
  if (world < 1 || world > kXMaxWorld) return fail(B2_ERR_ARG, "world must be in [1, %d]", kXMaxWorld);
  if (rank < 0 || rank >= world) return fail(B2_ERR_ARG, "rank must be in [0, world)");
  if (!areas || !dev_err) return fail(B2_ERR_ARG, "null pointer argument");
  XchgArgs x{nullptr, nullptr, batch, world, rank, out, dev_err, {}, poll_limit()};
  for (int r = 0; r < world; ++r) {
    if (!areas[r] || (reinterpret_cast<uintptr_t>(areas[r]) & 15))
      return fail(B2_ERR_ARG, "exchange area %d is null or not 16-byte aligned", r);
    x.area[r] = static_cast<char *>(areas[r]);
  }
  return decode_step_impl(qkv, row_stride, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_lens, seq_lens,
                          block_tables, max_blocks_per_seq, k_pool, v_pool, num_blocks, batch, blocks_per_split,
                          scale, mode, out, q_out, nullptr, nullptr, part_ml, part_o, counters, max_ctas, dev_err,
                          stream, &x);
}

extern "C" int b2_merge_states(const float *states, int32_t num_parts, int32_t batch, uint16_t *out,
                               float *state_ml, float *state_o, void *stream) {
  if (batch < 0) return fail(B2_ERR_ARG, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return ok();
  if (!states || num_parts <= 0) return fail(B2_ERR_ARG, "states and num_parts > 0 required");
  if (!out && !state_o) return fail(B2_ERR_ARG, "one of out or state_o is required");
  if ((state_o == nullptr) != (state_ml == nullptr)) return fail(B2_ERR_ARG, "state_ml and state_o go together");
  const int64_t part = static_cast<int64_t>(batch) * kHq * (2 + kDim);  // floats per part
  CombineArgs a{states, states + static_cast<int64_t>(batch) * kHq * 2, num_parts, nullptr, 1, out, state_ml,
                state_o, 0, 0, 0, kHq * 2, part, kHq * kDim, part, combine_groups(num_parts)};
  combine_kernel<<<dim3(batch, kHq), a.groups * kDim, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("combine_kernel (merge states)");
}

bool prefill_smem_ready() {
  static std::atomic<bool> done[128];  // per device; several host threads may launch at once
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return false;
  if (!done[dev]) {
    if (cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem) !=
        cudaSuccess)
      return false;
    done[dev] = true;
  }
  return true;
}

extern "C" int b2_prefill_append(const uint16_t *qkv, int64_t row_stride, const uint16_t *gamma_q,
                                 const uint16_t *gamma_k, float eps, const uint16_t *rope_cos,
                                 const uint16_t *rope_sin, int32_t rope_rows, const int32_t *past_lens,
                                 const int32_t *chunk_lens, int32_t tokens, const int32_t *block_tables,
                                 int32_t max_blocks_per_seq, uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks,
                                 uint16_t *q_out, int32_t batch, int32_t mode, int32_t *dev_err, void *stream) {
  if (batch < 0 || tokens < 0) return fail(B2_ERR_ARG, "batch and tokens must be >= 0");
  if (batch == 0 || tokens == 0) return ok();
  if (tokens > 65535) return fail(B2_ERR_ARG, "tokens must be <= 65535");
  if (!qkv || !past_lens || !dev_err) return fail(B2_ERR_ARG, "qkv, past_lens and dev_err are required");
  if (mode & ~(B2_NORM_QK | B2_ROPE_QK | B2_STORE_KV)) return fail(B2_ERR_ARG, "unknown mode bits 0x%x", mode);
  if (row_stride < kQkvWidth || row_stride % 8 != 0)
    return fail(B2_ERR_ARG, "row_stride must be >= %d and a multiple of 8", kQkvWidth);
  if (!aligned16(qkv) || (q_out && !aligned16(q_out))) return fail(B2_ERR_ARG, "qkv and q_out must be 16-byte aligned");
  if ((mode & B2_NORM_QK) && (!gamma_q || !gamma_k || !aligned16(gamma_q) || !aligned16(gamma_k)))
    return fail(B2_ERR_ARG, "B2_NORM_QK needs 16-byte aligned gamma_q and gamma_k");
  if ((mode & B2_ROPE_QK) &&
      (!rope_cos || !rope_sin || rope_rows <= 0 || !aligned16(rope_cos) || !aligned16(rope_sin)))
    return fail(B2_ERR_ARG, "B2_ROPE_QK needs 16-byte aligned cos/sin tables with rope_rows > 0");
  if (max_blocks_per_seq > kMaxTableWidth) return table_width_error(max_blocks_per_seq);
  if (mode & B2_STORE_KV) {
    if (!block_tables || !k_pool || !v_pool || max_blocks_per_seq <= 0 || num_blocks <= 0)
      return fail(B2_ERR_ARG, "B2_STORE_KV needs block_tables, k_pool, v_pool and positive sizes");
    if (!aligned16(k_pool) || !aligned16(v_pool)) return fail(B2_ERR_ARG, "pools must be 16-byte aligned");
  }
  AppendArgs a{qkv, row_stride, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_lens,
               block_tables, max_blocks_per_seq > 0 ? max_blocks_per_seq : 1, k_pool, v_pool,
               num_blocks, q_out, mode, dev_err, tokens, chunk_lens};
  append_rope_kernel<<<dim3(batch, tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_status("append_rope_kernel (chunk)");
}

extern "C" int b2_prefill_attn(const uint16_t *q, const uint16_t *k_pool, const uint16_t *v_pool, int32_t num_blocks,
                               const int32_t *block_tables, int32_t max_blocks_per_seq, const int32_t *past_lens,
                               const int32_t *chunk_lens, int32_t tokens, int32_t batch, float scale, uint16_t *out,
                               int32_t *dev_err, void *stream) {
  if (batch < 0 || tokens < 0) return fail(B2_ERR_ARG, "batch and tokens must be >= 0");
  if (batch == 0 || tokens == 0) return ok();
  if (!q || !k_pool || !v_pool || !block_tables || !past_lens || !out || !dev_err)
    return fail(B2_ERR_ARG, "null pointer argument");
  if (num_blocks <= 0 || static_cast<int64_t>(num_blocks) * kHkv * kBlock >= (int64_t(1) << 31))
    return fail(B2_ERR_ARG, "num_blocks must be in [1, 2^22) (got %d)", num_blocks);
  if (max_blocks_per_seq <= 0) return fail(B2_ERR_ARG, "max_blocks_per_seq must be positive");
  if (max_blocks_per_seq > kMaxTableWidth) return table_width_error(max_blocks_per_seq);
  if (batch > 65535) return fail(B2_ERR_ARG, "batch must be <= 65535");
  if (!aligned16(q) || !aligned16(out) || !aligned16(k_pool) || !aligned16(v_pool))
    return fail(B2_ERR_ARG, "q, out and the pools must be 16-byte aligned");
  if (!(scale > 0.f)) return fail(B2_ERR_ARG, "scale must be positive");
  CUtensorMap mk, mv;
  int rc = make_pool_map(&mk, k_pool, num_blocks);
  if (rc) return rc;
  rc = make_pool_map(&mv, v_pool, num_blocks);
  if (rc) return rc;
  if (!prefill_smem_ready()) return fail(B2_ERR_CUDA, "cannot set the prefill kernel's shared memory size");
  PrefillArgs a{q, block_tables, max_blocks_per_seq, past_lens, chunk_lens, tokens, num_blocks,
                scale * 1.4426950408889634f, out, dev_err, 0, 0, nullptr, nullptr, wait_limit()};
  const dim3 grid((tokens + 63) / 64, kHkv, batch);
  prefill_attn_kernel<<<grid, kPfThreads, kPfSmem, static_cast<cudaStream_t>(stream)>>>(mk, mv, a);
  return launch_status("prefill_attn_kernel");
}

extern "C" int b2_prefill_attn_split(const uint16_t *q, const uint16_t *k_pool, const uint16_t *v_pool,
                                     int32_t num_blocks, const int32_t *block_tables, int32_t max_blocks_per_seq,
                                     const int32_t *past_lens, const int32_t *chunk_lens, int32_t tokens,
                                     int32_t batch, float scale, int32_t blocks_per_split, float *part_ml,
                                     float *part_o, uint16_t *out, int32_t *dev_err, void *stream) {
  if (batch < 0 || tokens < 0) return fail(B2_ERR_ARG, "batch and tokens must be >= 0");
  if (batch == 0 || tokens == 0) return ok();
  if (!q || !k_pool || !v_pool || !block_tables || !past_lens || !out || !dev_err || !part_ml || !part_o)
    return fail(B2_ERR_ARG, "null pointer argument");
  if (num_blocks <= 0 || static_cast<int64_t>(num_blocks) * kHkv * kBlock >= (int64_t(1) << 31))
    return fail(B2_ERR_ARG, "num_blocks must be in [1, 2^22) (got %d)", num_blocks);
  if (max_blocks_per_seq <= 0) return fail(B2_ERR_ARG, "max_blocks_per_seq must be positive");
  if (max_blocks_per_seq > kMaxTableWidth) return table_width_error(max_blocks_per_seq);
  if (blocks_per_split <= 0 || blocks_per_split > kMaxTableWidth)
    return fail(B2_ERR_ARG, "blocks_per_split must be in [1, %d]", kMaxTableWidth);
  const int64_t nsplit = (static_cast<int64_t>(max_blocks_per_seq) + blocks_per_split - 1) / blocks_per_split;
  if (static_cast<int64_t>(batch) * nsplit > 65535) return fail(B2_ERR_ARG, "batch x splits must be <= 65535");
  if (static_cast<int64_t>(batch) * tokens * nsplit * kHq * kDim >= (int64_t(1) << 40))
    return fail(B2_ERR_ARG, "partial-state buffers too large");
  if (!aligned16(q) || !aligned16(out) || !aligned16(k_pool) || !aligned16(v_pool) || !aligned16(part_o) ||
      (reinterpret_cast<uintptr_t>(part_ml) & 7))
    return fail(B2_ERR_ARG, "q, out, the pools and part_o must be 16-byte aligned, part_ml 8-byte aligned");
  if (!(scale > 0.f)) return fail(B2_ERR_ARG, "scale must be positive");
  CUtensorMap mk, mv;
  int rc = make_pool_map(&mk, k_pool, num_blocks);
  if (rc) return rc;
  rc = make_pool_map(&mv, v_pool, num_blocks);
  if (rc) return rc;
  if (!prefill_smem_ready()) return fail(B2_ERR_CUDA, "cannot set the prefill kernel's shared memory size");
  PrefillArgs a{q, block_tables, max_blocks_per_seq, past_lens, chunk_lens, tokens, num_blocks,
                scale * 1.4426950408889634f, out, dev_err, blocks_per_split, static_cast<int>(nsplit),
                part_ml, part_o, wait_limit()};
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((tokens + 63) / 64, kHkv, static_cast<unsigned>(batch * nsplit));
  prefill_attn_kernel<<<grid, kPfThreads, kPfSmem, st>>>(mk, mv, a);
  rc = launch_status("prefill_attn_kernel (split)");
  if (rc) return rc;
  // merge the splits of every (sequence, token, head): rows b * tokens + t
  const int64_t rows = static_cast<int64_t>(batch) * tokens;
  if (rows > 0x7fffffff) return fail(B2_ERR_ARG, "batch x tokens too large");
  const int64_t ml_s = rows * kHq * 2, o_s = rows * kHq * kDim;
  CombineArgs c{part_ml, part_o, static_cast<int>(nsplit), nullptr, 1, out, nullptr, nullptr, 0, 0, 0,
                kHq * 2, ml_s, kHq * kDim, o_s, combine_groups(static_cast<int>(nsplit))};
  combine_kernel<<<dim3(static_cast<unsigned>(rows), kHq), c.groups * kDim, 0, st>>>(c);
  return launch_status("combine_kernel (prefill splits)");
}

extern "C" int b2_decode_step_host(const uint16_t *qkv_host, const int32_t *past_host, uint16_t *out_host,
                                   uint16_t *qkv_dev, int32_t *past_dev, uint16_t *out_dev, const uint16_t *gamma_q,
                                   const uint16_t *gamma_k, float eps, const uint16_t *rope_cos,
                                   const uint16_t *rope_sin, int32_t rope_rows, const int32_t *block_tables,
                                   int32_t max_blocks_per_seq, uint16_t *k_pool, uint16_t *v_pool, int32_t num_blocks,
                                   int32_t batch, int32_t blocks_per_split, float scale, float *part_ml, float *part_o,
                                   int32_t *counters, int32_t *dev_err, void *stream) {
  if (batch <= 0) return batch == 0 ? ok() : fail(B2_ERR_ARG, "batch must be >= 0");
  if (!qkv_host || !past_host || !out_host || !qkv_dev || !past_dev || !out_dev)
    return fail(B2_ERR_ARG, "null host or staging pointer");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t qkv_bytes = static_cast<size_t>(batch) * kQkvWidth * 2;
  const size_t out_bytes = static_cast<size_t>(batch) * kHq * kDim * 2;
  if (cudaMemcpyAsync(qkv_dev, qkv_host, qkv_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(past_dev, past_host, static_cast<size_t>(batch) * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return fail(B2_ERR_CUDA, "host-to-device copy failed: %s", cudaGetErrorString(cudaGetLastError()));
  const int rc = b2_decode_step(qkv_dev, kQkvWidth, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_dev,
                                nullptr, block_tables, max_blocks_per_seq, k_pool, v_pool, num_blocks, batch,
                                blocks_per_split, scale, B2_NORM_QK | B2_ROPE_QK | B2_STORE_KV, out_dev, nullptr,
                                nullptr, nullptr, part_ml, part_o, counters, 0, dev_err, stream);
  if (rc) return rc;
  if (cudaMemcpyAsync(out_host, out_dev, out_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return fail(B2_ERR_CUDA, "device-to-host copy failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

namespace {

// Streams and events of the double-buffered host-fed step, one set per device
// (created on first use; no device memory is allocated).
struct HostPipe {
  bool ready = false;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t in_ready[2] = {}, out_ready[2] = {}, slot_free[2] = {}, d2h_done = nullptr;
};
std::mutex g_pipe_mu;
HostPipe g_pipe[128];

HostPipe *host_pipe(int *rc) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) {
    *rc = fail(B2_ERR_CUDA, "no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  HostPipe &p = g_pipe[dev];
  if (!p.ready) {
    bool okk = cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking) == cudaSuccess &&
               cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking) == cudaSuccess &&
               cudaEventCreateWithFlags(&p.d2h_done, cudaEventDisableTiming) == cudaSuccess;
    for (int i = 0; i < 2 && okk; ++i)
      okk = cudaEventCreateWithFlags(&p.in_ready[i], cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&p.out_ready[i], cudaEventDisableTiming) == cudaSuccess &&
            cudaEventCreateWithFlags(&p.slot_free[i], cudaEventDisableTiming) == cudaSuccess &&
            cudaEventRecord(p.slot_free[i], p.d2h) == cudaSuccess;
    if (!okk) {
      *rc = fail(B2_ERR_CUDA, "cannot create the host pipeline's streams/events: %s",
                 cudaGetErrorString(cudaGetLastError()));
      return nullptr;
    }
    p.ready = true;
  }
  *rc = B2_OK;
  return &p;
}

}  // namespace

extern "C" int b2_decode_step_host2(const uint16_t *qkv_host, const int32_t *past_host, uint16_t *out_host,
                                    uint16_t *qkv_dev2, int32_t *past_dev2, uint16_t *out_dev2, int32_t slot,
                                    const uint16_t *gamma_q, const uint16_t *gamma_k, float eps,
                                    const uint16_t *rope_cos, const uint16_t *rope_sin, int32_t rope_rows,
                                    const int32_t *block_tables, int32_t max_blocks_per_seq, uint16_t *k_pool,
                                    uint16_t *v_pool, int32_t num_blocks, int32_t batch, int32_t blocks_per_split,
                                    float scale, float *part_ml, float *part_o, int32_t *counters,
                                    int32_t *dev_err, void *stream) {
  if (batch <= 0) return batch == 0 ? ok() : fail(B2_ERR_ARG, "batch must be >= 0");
  if (slot != 0 && slot != 1) return fail(B2_ERR_ARG, "slot must be 0 or 1");
  if (!qkv_host || !past_host || !out_host || !qkv_dev2 || !past_dev2 || !out_dev2)
    return fail(B2_ERR_ARG, "null host or staging pointer");
  int rc = B2_OK;
  HostPipe *p = host_pipe(&rc);
  if (!p) return rc;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t qkv_n = static_cast<size_t>(batch) * kQkvWidth, out_n = static_cast<size_t>(batch) * kHq * kDim;
  uint16_t *qkv_dev = qkv_dev2 + slot * qkv_n;
  int32_t *past_dev = past_dev2 + slot * batch;
  uint16_t *out_dev = out_dev2 + slot * out_n;
  // inputs: H2D on the pipeline's upload stream once the slot's previous use has finished
  if (cudaStreamWaitEvent(p->h2d, p->slot_free[slot], 0) != cudaSuccess ||
      cudaMemcpyAsync(qkv_dev, qkv_host, qkv_n * 2, cudaMemcpyHostToDevice, p->h2d) != cudaSuccess ||
      cudaMemcpyAsync(past_dev, past_host, static_cast<size_t>(batch) * 4, cudaMemcpyHostToDevice, p->h2d) !=
          cudaSuccess ||
      cudaEventRecord(p->in_ready[slot], p->h2d) != cudaSuccess || cudaStreamWaitEvent(st, p->in_ready[slot], 0) !=
                                                                        cudaSuccess)
    return fail(B2_ERR_CUDA, "host-to-device stage failed: %s", cudaGetErrorString(cudaGetLastError()));
  rc = b2_decode_step(qkv_dev, kQkvWidth, gamma_q, gamma_k, eps, rope_cos, rope_sin, rope_rows, past_dev, nullptr,
                      block_tables, max_blocks_per_seq, k_pool, v_pool, num_blocks, batch, blocks_per_split, scale,
                      B2_NORM_QK | B2_ROPE_QK | B2_STORE_KV, out_dev, nullptr, nullptr, nullptr, part_ml, part_o,
                      counters, 0, dev_err, stream);
  if (rc) return rc;
  // output: D2H on the download stream after the kernel; then the slot is free
  if (cudaEventRecord(p->out_ready[slot], st) != cudaSuccess ||
      cudaStreamWaitEvent(p->d2h, p->out_ready[slot], 0) != cudaSuccess ||
      cudaMemcpyAsync(out_host, out_dev, out_n * 2, cudaMemcpyDeviceToHost, p->d2h) != cudaSuccess ||
      cudaEventRecord(p->slot_free[slot], p->d2h) != cudaSuccess)
    return fail(B2_ERR_CUDA, "device-to-host stage failed: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

extern "C" int b2_decode_step_host_join(void *stream) {
  int rc = B2_OK;
  HostPipe *p = host_pipe(&rc);
  if (!p) return rc;
  if (cudaEventRecord(p->d2h_done, p->d2h) != cudaSuccess ||
      cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), p->d2h_done, 0) != cudaSuccess)
    return fail(B2_ERR_CUDA, "cannot join the host pipeline: %s", cudaGetErrorString(cudaGetLastError()));
  return ok();
}

namespace {

// ------------------------------------------------------------------ multi-GPU state exchange: standalone kernel, IPC

// grid (batch, 16 heads), block 64 threads (one per output dim).
__global__ void __launch_bounds__(kDim) exchange_merge_kernel(const XchgArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int bh = blockIdx.x * kHq + blockIdx.y, d = threadIdx.x;
  xchg_merge(a, blockIdx.x, blockIdx.y, d, a.state_ml[bh * 2], a.state_ml[bh * 2 + 1],
             a.state_o[(int64_t)bh * kDim + d]);
}

using PFN_memGetAddressRange = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

PFN_memGetAddressRange address_range_fn() {
  static const PFN_memGetAddressRange fn = [] {  // initialised once, thread-safe
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_memGetAddressRange>(p);
    return static_cast<PFN_memGetAddressRange>(nullptr);
  }();
  return fn;
}

}  // namespace

extern "C" int64_t b2_exchange_bytes(int32_t world, int32_t batch) {
  if (world < 1 || world > kXMaxWorld || batch < 1) return 0;
  return x_words(world, batch) * 8 + static_cast<int64_t>(batch) * kHq * 4;
}

extern "C" int b2_ipc_handle(const void *ptr, void *handle, int64_t *offset) {
  if (!ptr || !handle || !offset) return fail(B2_ERR_ARG, "null pointer argument");
  auto fn = address_range_fn();
  if (!fn) return fail(B2_ERR_NOSYM, "cuMemGetAddressRange is not available from the driver");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(B2_ERR_ARG, "pointer is not device memory of this context");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) return fail(B2_ERR_CUDA, "cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return ok();
}

extern "C" int b2_ipc_open(const void *handle, int64_t offset, void **peer_ptr) {
  if (!handle || !peer_ptr || offset < 0) return fail(B2_ERR_ARG, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(B2_ERR_CUDA, "cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
  *peer_ptr = static_cast<char *>(base) + offset;
  return ok();
}

extern "C" int b2_ipc_close(void *peer_ptr, int64_t offset) {
  if (!peer_ptr || offset < 0) return fail(B2_ERR_ARG, "bad argument");
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<char *>(peer_ptr) - offset);
  if (e != cudaSuccess) return fail(B2_ERR_CUDA, "cudaIpcCloseMemHandle failed: %s", cudaGetErrorString(e));
  return ok();
}

extern "C" int b2_exchange_merge(const float *state_ml, const float *state_o, int32_t batch, void *const *areas,
                                 int32_t world, int32_t rank, uint16_t *out, int32_t *dev_err, void *stream) {
  if (batch < 0) return fail(B2_ERR_ARG, "batch must be >= 0");
  if (batch == 0) return ok();
  if (batch > 65535) return fail(B2_ERR_ARG, "batch must be <= 65535");
  if (world < 1 || world > kXMaxWorld) return fail(B2_ERR_ARG, "world must be in [1, %d]", kXMaxWorld);
  if (rank < 0 || rank >= world) return fail(B2_ERR_ARG, "rank must be in [0, world)");
  if (!state_ml || !state_o || !areas || !out || !dev_err) return fail(B2_ERR_ARG, "null pointer argument");
  XchgArgs a{state_ml, state_o, batch, world, rank, out, dev_err, {}, poll_limit()};
  for (int r = 0; r < world; ++r) {
    if (!areas[r] || (reinterpret_cast<uintptr_t>(areas[r]) & 15))
      return fail(B2_ERR_ARG, "exchange area %d is null or not 16-byte aligned", r);
    a.area[r] = static_cast<char *>(areas[r]);
  }
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(batch), kHq);
  cfg.blockDim = dim3(kDim);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, exchange_merge_kernel, a) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    return fail(B2_ERR_CUDA, "exchange_merge_kernel launch failed: %s", cudaGetErrorString(e));
  }
  return launch_status("exchange_merge_kernel");
}

// ------------------------------------------------------------------ allocation-free decode

namespace {

constexpr int kNoAllocMlFloats = B2_NOALLOC_MAX_PARTS * kHq * 2;
constexpr int kNoAllocOFloats = B2_NOALLOC_MAX_PARTS * kHq * kDim;

// Partial states of b2_decode_attn_noalloc: [part_ml | part_o] for up to
// B2_NOALLOC_MAX_PARTS (sequence, split) pairs.  One copy per device.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocMlFloats + kNoAllocOFloats];

std::mutex g_noalloc_mu;
float *g_noalloc_ptr[128] = {};

// Device address of this device's scratch array.  Host code may not use the
// symbol itself (that names a host-side stand-in), so the address is looked
// up once per device with the device current.
float *noalloc_scratch(int *rc) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) {
    *rc = fail(B2_ERR_CUDA, "b2_decode_attn_noalloc: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *rc = fail(B2_ERR_CUDA, "b2_decode_attn_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(e));
      return nullptr;
    }
    g_noalloc_ptr[dev] = static_cast<float *>(p);
  }
  *rc = B2_OK;
  return g_noalloc_ptr[dev];
}

}  // namespace

extern "C" int b2_decode_attn_noalloc(const uint16_t *q, const uint16_t *k_pool, const uint16_t *v_pool,
                                      int32_t num_blocks, const int32_t *block_tables,
                                      int32_t max_blocks_per_seq, const int32_t *seq_lens, int32_t batch,
                                      int32_t blocks_per_split, float scale, uint16_t *out,
                                      int32_t *dev_err, void *stream) {
  if (batch < 0) return fail(B2_ERR_ARG, "batch must be >= 0 (got %d)", batch);
  if (batch == 0) return ok();
  if (!q || !k_pool || !v_pool || !block_tables || !seq_lens || !out || !dev_err)
    return fail(B2_ERR_ARG, "null pointer argument");
  if (max_blocks_per_seq <= 0 || blocks_per_split <= 0)
    return fail(B2_ERR_ARG, "max_blocks_per_seq and blocks_per_split must be positive");
  if (max_blocks_per_seq > kMaxTableWidth) return table_width_error(max_blocks_per_seq);
  if (blocks_per_split > kMaxTableWidth)
    return fail(B2_ERR_ARG, "blocks_per_split must be <= %d (got %d)", kMaxTableWidth, blocks_per_split);
  const int64_t splits = (static_cast<int64_t>(max_blocks_per_seq) + blocks_per_split - 1) / blocks_per_split;
  if (splits * batch > B2_NOALLOC_MAX_PARTS)
    return fail(B2_ERR_ARG,
                "b2_decode_attn_noalloc: batch * ceil(max_blocks_per_seq / blocks_per_split) = %lld exceeds "
                "the static scratch limit B2_NOALLOC_MAX_PARTS = %d; raise blocks_per_split or split the batch",
                (long long)(splits * batch), B2_NOALLOC_MAX_PARTS);
  if (splits * blocks_per_split * kBlock > 0x7fffffff)
    return fail(B2_ERR_ARG, "b2_decode_attn_noalloc: splits x blocks_per_split x 64 must fit an int32 token count");
  if (num_blocks <= 0 || static_cast<int64_t>(num_blocks) * kHkv * kBlock >= (int64_t(1) << 31))
    return fail(B2_ERR_ARG, "num_blocks must be in [1, 2^22) (got %d)", num_blocks);
  if (!aligned16(q) || !aligned16(k_pool) || !aligned16(v_pool))
    return fail(B2_ERR_ARG, "q and the pools must be 16-byte aligned");
  if (!(scale > 0.f)) return fail(B2_ERR_ARG, "scale must be positive");
  int rc = B2_OK;
  float *scratch = noalloc_scratch(&rc);
  if (!scratch) return rc;
  float *part_ml = scratch;
  float *part_o = scratch + kNoAllocMlFloats;
  CUtensorMap mk, mv;
  rc = make_pool_map(&mk, k_pool, num_blocks);
  if (rc) return rc;
  rc = make_pool_map(&mv, v_pool, num_blocks);
  if (rc) return rc;
  if (!decode_smem_ready()) return fail(B2_ERR_CUDA, "cannot set the decode kernel's shared memory size");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  DecodeArgs a{q, block_tables, max_blocks_per_seq, seq_lens, num_blocks, blocks_per_split,
               static_cast<int>(splits), scale * 1.4426950408889634f, part_ml, part_o, dev_err, wait_limit()};
  paged_decode_kernel<<<dim3(static_cast<unsigned>(splits), kHkv, batch), kDecodeThreads, kDecodeSmem, s>>>(mk, mv, a);
  rc = launch_status("paged_decode_kernel (noalloc)");
  if (rc) return rc;
  CombineArgs c{part_ml, part_o, static_cast<int>(splits), seq_lens, blocks_per_split, out, nullptr, nullptr,
                0, 0, static_cast<int>(splits) * blocks_per_split * kBlock, 0, 0, 0, 0,
                combine_groups(static_cast<int>(splits))};
  combine_kernel<<<dim3(batch, kHq), c.groups * kDim, 0, s>>>(c);
  return launch_status("combine_kernel (noalloc)");
}
