// B200 (sm_100a) projection GEMM of the LFM2.5 decode layer on the 5th-generation
// tensor cores:
//
//   gemm_kernel   D[m, n] = A[m, k] . W[n, k]^T, bf16 in, fp32 accumulate in TMEM,
//                 bf16 out; optional SwiGLU epilogue for the stacked w1 / w3
//                 weights (D = silu(A w1^T) * (A w3^T), the rounding points of
//                 the model's bf16 tensors).
//
// One CTA owns a 128-row x tile_n output tile over a slice of K.  Warp 0's lane
// 0 streams 64-wide K chunks of A and W into a ring of 128-byte-swizzled stages
// with TMA; warp 1's lane 0 issues tcgen05.mma (M 128, N = tile columns, K 16)
// into the TMEM accumulator and frees each stage with tcgen05.commit.  The
// weights do not depend on the previous kernel, so the first stages' W copies
// are issued before griddepcontrol.wait (programmatic dependent launch): they
// overlap the tail of the kernel that produces A.  Split-K runs the K slices
// of one tile as a thread-block cluster: every CTA stages its fp32 partial tile
// in its own shared memory, and CTA r of the cluster sums rows [r * 128 /
// splits, ...) of all partials over distributed shared memory in a fixed
// order (deterministic), applies the epilogue and stores bf16 rows.  No TMA
// multicast: every CTA loads its own tiles.
//
// The decode layer's projections are weight-streaming products (m = batch);
// the reference runs them as NPU GEMVs with fp32 accumulation and bf16 output
// (experiments/lfm25_bf16_gemv_kernel.py:19-60, the x8 engine's gemv_obj in
// experiments/kernels/x8/x8_core.cc:166-177) and as the projection halves of
// its attention prefix / tail programs (experiments/lfm25_attention_prefix_kernel.py,
// experiments/lfm25_attention_tail_kernel.py).

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>

#include <atomic>

#include "b2_block.h"
#include "b2_decode_attn.h"
#include "b2_internal.h"

namespace {

constexpr int kThreads = 128;  // 4 warps: producer lane, MMA lane, then all four run the epilogue
constexpr int kTileM = 128;    // UMMA M (one TMEM lane per tile row)
constexpr int kChunkK = 64;    // K elements per stage: one 128-byte swizzle row
constexpr uint32_t kATileBytes = kTileM * kChunkK * 2;  // 16 KiB
constexpr int kMaxStages = 8;
constexpr int kMaxSplits = 8;      // portable cluster size
constexpr int kMaxAccCols = 128;   // accumulator columns (tile_n, or 2 x tile_n for SwiGLU)
constexpr int kSmemBudget = 112 * 1024;  // two CTAs per SM
constexpr uint64_t kDrainNs = 2000000000ull;

struct GemmArgs {
  uint16_t *d;
  int64_t ldd;
  int m, n, k;
  int tile_n, splits, chunks, stages, mode;
  int32_t *err;
  uint64_t wait_ns;
};

struct GemmBars {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t done;
  uint32_t tmem;
};

__host__ __device__ constexpr int acc_cols(int tile_n, int mode) { return mode == B2_GEMM_SWIGLU ? 2 * tile_n : tile_n; }
__host__ __device__ constexpr uint32_t stage_bytes(int cols) { return kATileBytes + static_cast<uint32_t>(cols) * 128u; }
__host__ __device__ constexpr int part_bytes(int cols) { return kTileM * (cols + 4) * 4; }  // rows padded by 4 floats
__host__ __device__ constexpr uint32_t tmem_cols(int cols) { return cols <= 32 ? 32u : (cols <= 64 ? 64u : 128u); }

// ------------------------------------------------------------------ device helpers

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
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

// Wait for the phase of the given parity; false after limit_ns.
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

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void tma_load(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_hint(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar,
                                              uint64_t policy) {
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

// tcgen05 shared-memory descriptor: K-major, 128-byte swizzle, 128-byte rows,
// 8-row groups 1024 bytes apart, descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t r[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// float4 at a shared::cta address of cluster CTA `rank`
__device__ __forceinline__ float4 ld_peer4(uint32_t addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

__device__ __forceinline__ float4 ld_own4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// fp32 -> bf16 -> fp32, round to nearest even (torch's rounding)
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t bf16_pair(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}

// silu(g) * u at the model's bf16 rounding points (as b2_swiglu): g and u are
// the bf16 outputs of the two projections.
__device__ __forceinline__ float swiglu1(float g, float u) {
  g = bf16_round(g);
  u = bf16_round(u);
  return __fmul_rn(bf16_round(__fdiv_rn(g, 1.0f + expf(-g))), u);
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w, const GemmArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const bool swiglu = g.mode == B2_GEMM_SWIGLU;
  const int cols = acc_cols(g.tile_n, g.mode);
  const uint32_t sbytes = stage_bytes(cols);
  const int ring = g.stages * static_cast<int>(sbytes);
  GemmBars *bars = reinterpret_cast<GemmBars *>(smem + (ring > part_bytes(cols) ? ring : part_bytes(cols)));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t split = g.splits > 1 ? cluster_rank() : 0;
  const int m0 = static_cast<int>(blockIdx.x / g.splits) * kTileM;
  const int n0 = static_cast<int>(blockIdx.y) * g.tile_n;
  const int kc0 = static_cast<int>(split) * g.chunks;
  const uint32_t ncols = tmem_cols(cols);

  if (threadIdx.x == 0) {
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    mbar_init(smem_u32(&bars->done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = bars->tmem;

  if (warp == 0 && lane == 0) {
    // producer: the first stages' weight tiles go out before the wait for the
    // kernel that writes A; the activation tiles after it
    const uint64_t pol_w = evict_first_policy();
    const int pre = g.chunks < g.stages ? g.chunks : g.stages;
    for (int c = 0; c < pre; ++c) {
      const uint32_t full = smem_u32(&bars->full[c]);
      const uint32_t b = smem_u32(smem + c * sbytes + kATileBytes);
      const int x = (kc0 + c) * kChunkK;
      mbar_arrive_expect_tx(full, sbytes);
      tma_load_hint(b, &tm_w, x, n0, full, pol_w);
      if (swiglu) tma_load_hint(b + g.tile_n * 128, &tm_w, x, g.n + n0, full, pol_w);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int c = 0; c < pre; ++c)
      tma_load(smem_u32(smem + c * sbytes), &tm_a, (kc0 + c) * kChunkK, m0, smem_u32(&bars->full[c]));
    int issued = pre;
    for (int c = pre; c < g.chunks; ++c) {
      const int s = c % g.stages;
      if (!mbar_wait(smem_u32(&bars->empty[s]), ((c / g.stages) - 1) & 1, g.wait_ns)) {
        atomicOr(g.err, B2_DEV_TIMEOUT);
        break;
      }
      const uint32_t full = smem_u32(&bars->full[s]);
      const uint32_t a = smem_u32(smem + s * sbytes);
      const int x = (kc0 + c) * kChunkK;
      mbar_arrive_expect_tx(full, sbytes);
      tma_load_hint(a + kATileBytes, &tm_w, x, n0, full, pol_w);
      if (swiglu) tma_load_hint(a + kATileBytes + g.tile_n * 128, &tm_w, x, g.n + n0, full, pol_w);
      tma_load(a, &tm_a, x, m0, full);
      issued = c + 1;
    }
    // the CTA's shared memory must outlive every copy into it: wait (bounded)
    // until the last stages' copies have landed
    for (int c = issued - g.stages < 0 ? 0 : issued - g.stages; c < issued; ++c)
      if (!mbar_wait(smem_u32(&bars->full[c % g.stages]), (c / g.stages) & 1, kDrainNs)) atomicOr(g.err, B2_DEV_TIMEOUT);
  } else if (warp == 1 && lane == 0) {
    // f32 accumulator, bf16 A and B, both K-major, M 128, N = cols
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(cols >> 3) << 17) |
                           (static_cast<uint32_t>(kTileM >> 4) << 24);
    for (int c = 0; c < g.chunks; ++c) {
      const int s = c % g.stages;
      if (!mbar_wait(smem_u32(&bars->full[s]), (c / g.stages) & 1, g.wait_ns)) {
        atomicOr(g.err, B2_DEV_TIMEOUT);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a = smem_u32(smem + s * sbytes), b = a + kATileBytes;
#pragma unroll
      for (int kk = 0; kk < kChunkK / 16; ++kk)
        umma_bf16(tmem, umma_desc(a + 32 * kk), umma_desc(b + 32 * kk), idesc, (c | kk) != 0);
      umma_commit(smem_u32(&bars->empty[s]));
    }
    umma_commit(smem_u32(&bars->done));  // tracks every product issued above
  }
  __syncwarp();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // epilogue: TMEM lane = tile row = threadIdx.x; the fp32 partial tile goes
  // to this CTA's shared memory (the ring is idle once the products are done)
  if (!mbar_wait(smem_u32(&bars->done), 0, kDrainNs)) atomicOr(g.err, B2_DEV_TIMEOUT);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  float *part = reinterpret_cast<float *>(smem);
  const int pstride = cols + 4;
  {
    const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float4 *row = reinterpret_cast<float4 *>(part + threadIdx.x * pstride);
    for (int c0 = 0; c0 < cols; c0 += 16) {
      uint32_t r[16];
      tmem_ld16(taddr + c0, r);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        row[c0 / 4 + q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                      __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  if (g.splits > 1) cluster_sync(); else __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
  }

  // rows [split * R, split * R + R) of the tile: the splits' partials summed in
  // cluster-rank order, then the epilogue; 4 output columns per thread and step
  const int rows = kTileM / g.splits;
  const int quads = g.tile_n / 4;
  for (int i = threadIdx.x; i < rows * quads; i += kThreads) {
    const int r = static_cast<int>(split) * rows + i / quads;
    const int c4 = i - (i / quads) * quads;
    const uint32_t off = smem_u32(part + r * pstride + 4 * c4);
    const uint32_t off_u = off + 4u * g.tile_n;
    float4 s = g.splits > 1 ? ld_peer4(off, 0) : ld_own4(off);
    float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
    if (swiglu) u = g.splits > 1 ? ld_peer4(off_u, 0) : ld_own4(off_u);
    for (int q = 1; q < g.splits; ++q) {
      const float4 v = ld_peer4(off, q);
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      if (swiglu) {
        const float4 w = ld_peer4(off_u, q);
        u.x += w.x; u.y += w.y; u.z += w.z; u.w += w.w;
      }
    }
    if (swiglu) {
      s.x = swiglu1(s.x, u.x);
      s.y = swiglu1(s.y, u.y);
      s.z = swiglu1(s.z, u.z);
      s.w = swiglu1(s.w, u.w);
    }
    const int gr = m0 + r;
    if (gr < g.m)
      *reinterpret_cast<uint2 *>(g.d + static_cast<int64_t>(gr) * g.ldd + n0 + 4 * c4) =
          make_uint2(bf16_pair(s.x, s.y), bf16_pair(s.z, s.w));
  }
  __syncwarp();
  if (g.splits > 1) cluster_sync();  // the other CTAs read this CTA's partial until here
}

// ------------------------------------------------------------------ host side

int fail(int code, const char *msg) { return b2_record_error(code, msg); }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
  }();
  return fn;
}

// a row-major bf16 matrix [rows, k] with row stride ld, boxes of 64 x box_rows
bool make_map(CUtensorMap *map, const void *base, int64_t rows, int64_t k, int64_t ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kChunkK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

bool smem_ready() {
  static std::atomic<bool> done[128];  // per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 128) return false;
  if (!done[dev]) {
    if (cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 2048) !=
        cudaSuccess)
      return false;
    done[dev] = true;
  }
  return true;
}

struct Plan {
  int tile_n, splits, chunks, stages, smem, ctas;
};

// Tile width, K splits and ring depth for an m x n x k product.  Wider tiles
// read A fewer times (A is re-read once per column tile); K splits keep about
// one CTA per SM busy when the tiles are few.
bool plan_gemm(int m, int n, int k, int mode, int tile_n, int splits, int sms, Plan *p) {
  const int mt = (m + kTileM - 1) / kTileM;
  const int kch = k / kChunkK;
  const int max_tile = mode == B2_GEMM_SWIGLU ? kMaxAccCols / 2 : kMaxAccCols;
  if (tile_n <= 0) {
    tile_n = 0;
    const int cands[4] = {128, 64, 32, 16};
    for (int t : cands) {
      if (t > max_tile || n % t) continue;
      if (tile_n == 0) tile_n = t;  // the widest that divides n
      if (t == 128 && static_cast<int64_t>(mt) * (n / t) >= 2 * sms) { tile_n = t; break; }
      if (t <= 64) { tile_n = t; break; }
    }
    if (tile_n == 0) return false;
  }
  if (tile_n % 16 || tile_n > max_tile || n % tile_n) return false;
  const int64_t tiles = static_cast<int64_t>(mt) * (n / tile_n);
  if (splits <= 0) {
    splits = 1;
    while (splits * 2 <= kMaxSplits && tiles * splits * 2 <= (3 * sms) / 2 && kch % (splits * 2) == 0 &&
           kch / (splits * 2) >= 2)
      splits *= 2;
  }
  if (splits < 1 || splits > kMaxSplits || (splits & (splits - 1)) || kch % splits) return false;
  const int cols = acc_cols(tile_n, mode);
  const int chunks = kch / splits;
  int stages = (kSmemBudget - static_cast<int>(sizeof(GemmBars))) / static_cast<int>(stage_bytes(cols));
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages > chunks) stages = chunks;
  if (stages < 1) return false;
  const int ring = stages * static_cast<int>(stage_bytes(cols));
  const int body = ring > part_bytes(cols) ? ring : part_bytes(cols);
  p->tile_n = tile_n;
  p->splits = splits;
  p->chunks = chunks;
  p->stages = stages;
  p->smem = body + static_cast<int>(sizeof(GemmBars)) + 1024;
  p->ctas = static_cast<int>(tiles * splits);
  return p->smem <= kSmemBudget + 2048;
}

int launch_error(const char *what) {
  const cudaError_t e = cudaGetLastError();
  char msg[256];
  snprintf(msg, sizeof(msg), "b2_gemm: %s: %s", what, cudaGetErrorString(e));
  return fail(B2_ERR_CUDA, msg);
}

}  // namespace

extern "C" int b2_gemm_plan(int32_t m, int32_t n, int32_t k, int32_t mode, int32_t *tile_n, int32_t *splits,
                            int32_t *ctas) {
  if (!tile_n || !splits) return fail(B2_ERR_ARG, "b2_gemm_plan: null pointer argument");
  Plan p{};
  if (m <= 0 || n <= 0 || k <= 0 || k % kChunkK || (mode != B2_GEMM_PLAIN && mode != B2_GEMM_SWIGLU) ||
      !plan_gemm(m, n, k, mode, *tile_n, *splits, sm_count(), &p))
    return fail(B2_ERR_ARG, "b2_gemm_plan: unsupported shape, mode, tile_n or splits");
  *tile_n = p.tile_n;
  *splits = p.splits;
  if (ctas) *ctas = p.ctas;
  return b2_clear_error();
}

extern "C" int b2_gemm(const uint16_t *a, int64_t lda, const uint16_t *w, int64_t ldw, uint16_t *d, int64_t ldd,
                       int32_t m, int32_t n, int32_t k, int32_t mode, int32_t tile_n, int32_t splits,
                       int32_t *dev_err, void *stream) {
  if (m < 0 || n < 0 || k < 0) return fail(B2_ERR_ARG, "b2_gemm: sizes must be >= 0");
  if (m == 0 || n == 0) return b2_clear_error();
  if (!a || !w || !d || !dev_err) return fail(B2_ERR_ARG, "b2_gemm: null pointer argument");
  if (mode != B2_GEMM_PLAIN && mode != B2_GEMM_SWIGLU) return fail(B2_ERR_ARG, "b2_gemm: unknown mode");
  if (k == 0 || k % kChunkK) return fail(B2_ERR_ARG, "b2_gemm: k must be a positive multiple of 64");
  if (!aligned16(a) || !aligned16(w) || !aligned16(d))
    return fail(B2_ERR_ARG, "b2_gemm: a, w and d must be 16-byte aligned");
  if (lda < k || ldw < k || lda % 8 || ldw % 8)
    return fail(B2_ERR_ARG, "b2_gemm: lda and ldw must be >= k and multiples of 8");
  if (ldd < n || ldd % 8) return fail(B2_ERR_ARG, "b2_gemm: ldd must be >= n and a multiple of 8");
  if ((static_cast<int64_t>(m) + kTileM - 1) / kTileM * kMaxSplits > 0x7fffffff)
    return fail(B2_ERR_ARG, "b2_gemm: m too large");
  Plan p{};
  if (!plan_gemm(m, n, k, mode, tile_n, splits, sm_count(), &p))
    return fail(B2_ERR_ARG,
                "b2_gemm: no tiling for this shape (tile_n must divide n, be a multiple of 16 and <= 128, "
                "or <= 64 with SwiGLU; splits a power of two <= 8 dividing k / 64)");
  if (n / p.tile_n > 65535) return fail(B2_ERR_ARG, "b2_gemm: n / tile_n must be <= 65535");
  CUtensorMap ma, mw;
  const int64_t wrows = mode == B2_GEMM_SWIGLU ? 2 * static_cast<int64_t>(n) : n;
  if (!make_map(&ma, a, m, k, lda, kTileM) || !make_map(&mw, w, wrows, k, ldw, p.tile_n))
    return fail(B2_ERR_NOSYM, "b2_gemm: cuTensorMapEncodeTiled is not available or refused the operands");
  if (!smem_ready()) return fail(B2_ERR_CUDA, "b2_gemm: cannot set the kernel's shared-memory size");
  GemmArgs g{d, ldd, m, n, k, p.tile_n, p.splits, p.chunks, p.stages, mode, dev_err, b2_wait_limit_ns()};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((m + kTileM - 1) / kTileM * p.splits), static_cast<unsigned>(n / p.tile_n));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(p.smem);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attrs[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  if (p.splits > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = static_cast<unsigned>(p.splits);
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  if (cudaLaunchKernelEx(&cfg, gemm_kernel, ma, mw, g) != cudaSuccess) return launch_error("gemm_kernel launch failed");
  if (cudaPeekAtLastError() != cudaSuccess) return launch_error("gemm_kernel launch failed");
  return b2_clear_error();
}
