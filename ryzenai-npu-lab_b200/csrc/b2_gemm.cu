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
// overlap the tail of the kernel that produces A (the layer kernels of
// b2_block.cu allow it from their first instruction).  Without a K split each
// thread converts its TMEM row and stores it.  Split-K runs the K slices of
// one tile as a thread-block cluster: every CTA stages its fp32 partial tile
// in its own shared memory and sends rows [r * 128 / splits, ...) to cluster
// CTA r with a bulk shared-to-shared copy (point to point, completing on the
// receiver's mbarrier); CTA r sums the slices of its rows in K-slice order
// (deterministic), applies the epilogue and stores bf16 rows.  No TMA
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
constexpr int kMaxStages = 16;
constexpr int kMaxSplits = 8;      // portable cluster size
constexpr int kMaxAccCols = 128;   // accumulator columns (tile_n, or 2 x tile_n for SwiGLU)
constexpr int kSmemBudget = 112 * 1024;      // two CTAs per SM
constexpr int kSmemBudgetOne = 200 * 1024;   // one CTA per SM (grids of at most one CTA per SM)
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
  uint64_t recv;  // split K: the other K slices' rows of this CTA have landed
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

__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t r[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// shared::cluster address of the same shared-memory offset in cluster CTA `rank`
__device__ __forceinline__ uint32_t peer_addr(uint32_t addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(addr), "r"(rank));
  return remote;
}

// Bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory into
// another cluster CTA's, completing on that CTA's mbarrier (point to point).
__device__ __forceinline__ void push_to_peer(uint32_t dst_cluster, uint32_t src, uint32_t bytes,
                                             uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst_cluster),
               "r"(src), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

__device__ __forceinline__ float4 ld_smem4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

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
  // [ring (reused for this CTA's fp32 partial tile) | split K: receive area,
  // the same [128][cols + 4] layout, rows r * R.. from K slice r | barriers]
  const int body = ring > part_bytes(cols) ? ring : part_bytes(cols);
  float *recv = reinterpret_cast<float *>(smem + body);
  GemmBars *bars = reinterpret_cast<GemmBars *>(smem + body + (g.splits > 1 ? part_bytes(cols) : 0));
  const int rows_per_split = kTileM / g.splits;
  const uint32_t slice_bytes = static_cast<uint32_t>(rows_per_split * (cols + 4) * 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t split = g.splits > 1 ? cluster_rank() : 0;
  const int m0 = static_cast<int>(blockIdx.x / g.splits) * kTileM;
  const int n0 = static_cast<int>(blockIdx.y) * g.tile_n;
  const int kc0 = static_cast<int>(split) * g.chunks;
  const uint32_t ncols = tmem_cols(cols);

  if (threadIdx.x == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_a)) : "memory");
    for (int s = 0; s < g.stages; ++s) {
      mbar_init(smem_u32(&bars->full[s]), 1);
      mbar_init(smem_u32(&bars->empty[s]), 1);
    }
    mbar_init(smem_u32(&bars->done), 1);
    if (g.splits > 1) {
      mbar_init(smem_u32(&bars->recv), 1);
      // the other splits' slices of this CTA's rows, pushed by their CTAs
      mbar_arrive_expect_tx(smem_u32(&bars->recv), static_cast<uint32_t>(g.splits - 1) * slice_bytes);
    }
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
  // phase 1 of the cluster barrier: this CTA's receive barrier is set up (the
  // wait comes just before the first push, long after every CTA arrived)
  if (g.splits > 1) cluster_arrive_relaxed();

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

  // epilogue: TMEM lane = tile row = threadIdx.x
  if (!mbar_wait(smem_u32(&bars->done), 0, kDrainNs)) atomicOr(g.err, B2_DEV_TIMEOUT);
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int grow = m0 + static_cast<int>(threadIdx.x);

  if (g.splits == 1) {
    // one K slice: each thread converts its own row and stores it, 16
    // columns (32 bytes) at a time; no shared memory, no barrier
    uint16_t *drow = g.d + static_cast<int64_t>(grow) * g.ldd + n0;
    for (int c0 = 0; c0 < g.tile_n; c0 += 16) {
      uint32_t r[16], ru[16];
      tmem_ld16_nowait(taddr + c0, r);
      if (swiglu) tmem_ld16_nowait(taddr + g.tile_n + c0, ru);
      tmem_wait_ld();
      uint32_t w[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float lo = __uint_as_float(r[2 * q]), hi = __uint_as_float(r[2 * q + 1]);
        if (swiglu) {
          lo = swiglu1(lo, __uint_as_float(ru[2 * q]));
          hi = swiglu1(hi, __uint_as_float(ru[2 * q + 1]));
        }
        w[q] = bf16_pair(lo, hi);
      }
      if (grow < g.m) {
        reinterpret_cast<uint4 *>(drow + c0)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4 *>(drow + c0)[1] = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
    }
    return;
  }

  // split K: the fp32 partial tile goes to this CTA's shared memory (the ring
  // is idle once the products are done), padded rows of cols + 4 floats
  float *part = reinterpret_cast<float *>(smem);
  const int pstride = cols + 4;
  {
    float4 *row = reinterpret_cast<float4 *>(part + threadIdx.x * pstride);
    for (int c0 = 0; c0 < cols; c0 += 32) {
      uint32_t r[32];
      tmem_ld16_nowait(taddr + c0, r);
      if (c0 + 16 < cols) tmem_ld16_nowait(taddr + c0 + 16, r + 16);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (c0 + 4 * q < cols)
          row[c0 / 4 + q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                        __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
    }
  }
  // the partial tile is read next by the bulk-copy (async) proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols));
  }
  cluster_wait();  // phase 1: every CTA's receive barrier is initialised
  const int rows = rows_per_split;
  if (threadIdx.x == 0) {
    // rows [q * R, q * R + R) of this partial go to CTA q, into its slot `split`
    for (int q = 0; q < g.splits; ++q) {
      if (q == static_cast<int>(split)) continue;
      push_to_peer(peer_addr(smem_u32(recv + split * rows * pstride), q), smem_u32(part + q * rows * pstride),
                   slice_bytes, peer_addr(smem_u32(&bars->recv), q));
    }
  }
  if (!mbar_wait(smem_u32(&bars->recv), 0, g.wait_ns)) atomicOr(g.err, B2_DEV_TIMEOUT);
  // phase 2: all pushes into this CTA have landed; when every CTA has arrived,
  // every push out of this CTA has been read and its partial may go
  cluster_arrive_relaxed();

  // rows [split * R, split * R + R) of the tile: the slices summed in K-slice
  // order (this CTA's own slice from its partial tile), then the epilogue.
  // Thread t keeps column quad t % quads and takes rows t / quads + j *
  // (128 / quads): four rows per round, their loads of a slice issued together.
  const int quads = g.tile_n / 4;                  // a power of two (tile_n is 16, 32, 64 or 128)
  const int qshift = __ffs(quads) - 1;
  const int step = kThreads >> qshift;             // rows per pass of the CTA
  const int c = 4 * (static_cast<int>(threadIdx.x) & (quads - 1));
  const int lr0 = static_cast<int>(threadIdx.x) >> qshift;
  for (int base = lr0; base < rows; base += 4 * step) {
    float4 sm[4], u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) sm[e] = u[e] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int q = 0; q < g.splits; ++q) {
      const float *slice = q == static_cast<int>(split) ? part + split * rows * pstride : recv + q * rows * pstride;
      float4 v[4], w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int lr = base + e * step;
        if (lr < rows) {
          v[e] = ld_smem4(slice + lr * pstride + c);
          if (swiglu) w[e] = ld_smem4(slice + lr * pstride + g.tile_n + c);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (base + e * step < rows) {
          sm[e].x += v[e].x; sm[e].y += v[e].y; sm[e].z += v[e].z; sm[e].w += v[e].w;
          if (swiglu) { u[e].x += w[e].x; u[e].y += w[e].y; u[e].z += w[e].z; u[e].w += w[e].w; }
        }
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int lr = base + e * step;
      if (lr >= rows) break;
      float4 o = sm[e];
      if (swiglu) {
        o.x = swiglu1(o.x, u[e].x);
        o.y = swiglu1(o.y, u[e].y);
        o.z = swiglu1(o.z, u[e].z);
        o.w = swiglu1(o.w, u[e].w);
      }
      const int gr = m0 + static_cast<int>(split) * rows + lr;
      if (gr < g.m)
        *reinterpret_cast<uint2 *>(g.d + static_cast<int64_t>(gr) * g.ldd + n0 + c) =
            make_uint2(bf16_pair(o.x, o.y), bf16_pair(o.z, o.w));
    }
  }
  __syncwarp();
  cluster_wait();  // phase 2
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
    if (cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudgetOne + 2048) !=
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
// one CTA per SM busy when the tiles are few.  A grid that leaves every CTA an
// SM of its own gets a deeper ring (the loop is bound by in-flight bytes /
// latency); split K also needs a receive area for the other slices' rows.
bool plan_gemm(int m, int n, int k, int mode, int tile_n, int splits, int sms, Plan *p) {
  const int mt = (m + kTileM - 1) / kTileM;
  const int kch = k / kChunkK;
  const int max_tile = mode == B2_GEMM_SWIGLU ? kMaxAccCols / 2 : kMaxAccCols;
  if (tile_n <= 0) {
    tile_n = 0;
    // 128 columns when that alone fills the GPU twice (the vocabulary head);
    // else 32 (measured on the decode layer's shapes at m = 256: 32 beat 64
    // in four of five, with split K filling the SMs), else what divides n
    const int cands[4] = {128, 32, 64, 16};
    for (int t : cands) {
      if (t > max_tile || n % t) continue;
      if (t == 128 && static_cast<int64_t>(mt) * (n / t) < 2 * sms) continue;
      tile_n = t;
      break;
    }
    if (tile_n == 0) return false;
  }
  if (tile_n % 16 || tile_n > max_tile || n % tile_n) return false;
  const int64_t tiles = static_cast<int64_t>(mt) * (n / tile_n);
  const int cols = acc_cols(tile_n, mode);
  auto fit = [&](int sp, Plan *out) {
    if (sp < 1 || sp > kMaxSplits || (sp & (sp - 1)) || kch % sp) return false;
    const int chunks = kch / sp;
    const int budget = tiles * sp <= sms ? kSmemBudgetOne : kSmemBudget;
    const int recv = sp > 1 ? part_bytes(cols) : 0;
    int stages = (budget - recv - static_cast<int>(sizeof(GemmBars))) / static_cast<int>(stage_bytes(cols));
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages > chunks) stages = chunks;
    if (stages < 1) return false;
    const int ring = stages * static_cast<int>(stage_bytes(cols));
    const int body = ring > part_bytes(cols) ? ring : part_bytes(cols);
    out->tile_n = tile_n;
    out->splits = sp;
    out->chunks = chunks;
    out->stages = stages;
    out->smem = body + recv + static_cast<int>(sizeof(GemmBars)) + 1024;
    out->ctas = static_cast<int>(tiles * sp);
    return out->smem <= budget + 2048;
  };
  if (splits > 0) return fit(splits, p);
  int sp = 1;
  while (sp * 2 <= kMaxSplits && tiles * sp * 2 <= 2 * sms && kch % (sp * 2) == 0 && kch / (sp * 2) >= 2)
    sp *= 2;
  for (; sp >= 1; sp /= 2)
    if (fit(sp, p)) return true;
  return false;
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
