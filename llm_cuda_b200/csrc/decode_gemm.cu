// Decode GEMM on the 5th-generation tensor cores: y[Mb, N] = x[Mb, K] . W[N, K]^T.
//
// The projections of a decode step (q/k/v, o, gate/up, down, lm_head at batch
// Mb <= 256) stream their weights exactly once: the GEMM is HBM-bound on W.  Each
// CTA owns 128 output features (W rows) and a range of K:
//
//   warp 0      TMA producer: W tile [128 x 64] and x tile [NB x 64] per 64-wide
//               k-chunk (cp.async.bulk.tensor, 128-byte swizzle) into a ring of
//               stages, completion on "full" mbarriers with transaction bytes;
//   warp 1      allocates NB TMEM columns; one elected thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M = 128, N = NB, K = 16, bf16 in,
//               fp32 accumulate in TMEM) from shared-memory descriptors and returns
//               each stage with tcgen05.commit on its "empty" mbarrier;
//   warps 2-5   epilogue: tcgen05.ld 32x32b of their TMEM lane quarter (lane = output
//               feature, column = batch row), then bf16 stores.
//
// Work split, by shape:
//   * stream-K (N / 128 >= 74 tiles): CTA c takes units [c*W/G, (c+1)*W/G) of the
//     W = tiles * k-chunks units; a tile shared by several CTAs is summed from fp32
//     parts by the CTA that completes it (global slots + a self-resetting counter).
//   * cluster split-K (fewer tiles): a cluster of S CTAs (S <= 8) owns one tile, each
//     CTA a 1/S slice of K; the S accumulators are summed through distributed shared
//     memory behind two cluster barriers, with no global round trip.
// Programmatic dependent launch: the weights never depend on the previous kernel, so
// the first ring stages of W are requested before griddepcontrol.wait and only the
// activation loads (and every global write) wait for the predecessor.
//
// D = A . B^T with A = W tile (K-major), B = x tile (K-major), so D^T = y tile.
// Every mbarrier wait is bounded; TMEM is always released.
#include <string>

#include "common.cuh"

namespace llmc {
namespace gemm {

constexpr int kTileN = 128;            // output features per CTA (UMMA M)
constexpr int kChunk = 64;             // k elements per stage (one 128-byte swizzle row)
constexpr int kThreads = 192;

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  // K-major, 128-byte swizzle: start >> 4, LBO = 1 (16 B), SBO = 1024 B (8 rows of 128 B),
  // descriptor version 1 (sm_100), layout type 2 (SWIZZLE_128B).
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
         (2ull << 61);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 columns of fp32 from TMEM into 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

struct Params {
  __nv_bfloat16* y;    // [Mb, N]
  float* ws;           // [tiles][max_seg][NB][128] fp32 partial slots of shared tiles
  int32_t* counters;   // [N / 128], all zero between calls
  int32_t* status;
  int Mb, N, K;
  long long units;     // tiles * k-chunks
  int max_seg;         // slots per tile
  int cluster;         // cluster split-K: CTAs per tile (0: stream-K)
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}
__device__ __forceinline__ void st_dsmem_f32(uint32_t remote_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote_addr), "f"(v) : "memory");
}

// Ring depth that fits 227 KB of shared memory for a batch tile of NB rows.
template <int NB, int CPS>
struct Ring {
  static constexpr int kStageBytes = (kTileN + NB) * kChunk * 2 * CPS;
  static constexpr int kStages = (200 * 1024) / kStageBytes > 8 ? 8 : (200 * 1024) / kStageBytes;
};

// Stream-K split of units [0, W) over G CTAs: CTA c owns [start(c), start(c+1)).
__device__ __forceinline__ long long sk_start(long long c, long long W, long long G) {
  return c * W / G;
}
__device__ __forceinline__ int sk_owner(long long u, long long W, long long G) {
  long long c = u * G / W;
  while (c + 1 < G && sk_start(c + 1, W, G) <= u) ++c;
  while (c > 0 && sk_start(c, W, G) > u) --c;
  return (int)c;
}

// CPS consecutive 64-wide k-chunks per stage: each weight row contributes 128*CPS
// contiguous bytes per stage, which the DRAM serves far better than 128-byte pieces.
template <int NB, int CPS>
__global__ void __launch_bounds__(kThreads, 1)
decode_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, const Params p) {
  constexpr uint32_t A1 = kTileN * kChunk * 2;        // one W chunk box: 16 KB
  constexpr uint32_t B1 = NB * kChunk * 2;            // one x chunk box
  constexpr uint32_t A_BYTES = A1 * CPS;
  constexpr uint32_t B_BYTES = B1 * CPS;
  constexpr uint32_t STAGE = A_BYTES + B_BYTES;
  constexpr int kStages = Ring<NB, CPS>::kStages;
  // Instruction descriptor: fp32 accumulate, bf16 A and B, both K-major, N = NB, M = 128.
  constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(NB >> 3) << 17) |
                             ((uint32_t)(kTileN >> 4) << 24);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kStages * STAGE);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* tfull_bar = empty_bar + kStages;     // [2] accumulator ready
  uint64_t* tempty_bar = tfull_bar + 2;          // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KC = p.K / (kChunk * CPS);   // work units (stages) per tile
  const long long W = p.units, G = gridDim.x;
  const bool cl = p.cluster > 0;
  long long u0, u1;
  uint32_t crank = 0;
  if (cl) {   // cluster split-K: tile blockIdx.x / S, K slice of this CTA's cluster rank
    crank = cluster_ctarank();
    const long long tile = blockIdx.x / p.cluster;
    u0 = tile * KC + (long long)crank * KC / p.cluster;
    u1 = tile * KC + ((long long)crank + 1) * KC / p.cluster;
  } else {
    u0 = sk_start(blockIdx.x, W, G);
    u1 = sk_start(blockIdx.x + 1, W, G);
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull_bar[b]), 1);
      mbar_init(smem_u32(&tempty_bar[b]), 4);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {   // TMEM: two accumulators of NB fp32 columns x 128 lanes
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"((uint32_t)(2 * NB))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tmap_w);
    prefetch_tensormap(&tmap_x);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  pdl_launch_dependents();
  float acc_lo[32], acc_hi[32];   // cluster split-K: this thread's accumulator row
  if (warp == 0) {
    // ---- TMA producer: every k-chunk of this CTA's range, across tile boundaries ----
    if (lane == 0) {
      // The first ring-full of weight boxes goes out before waiting for the previous
      // kernel (weights are never written by it); the activation boxes follow the wait.
      const long long pre = (u1 - u0) < kStages ? (u1 - u0) : kStages;
      for (long long i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        const uint32_t fb = smem_u32(&full_bar[i]);
        mbar_arrive_expect_tx(fb, STAGE);
        const int tile = (int)(u / KC), kc = (int)(u % KC) * CPS;
        const uint32_t a = smem_u32(smem + i * STAGE);
#pragma unroll
        for (int j = 0; j < CPS; ++j) tma_load_2d(a + j * A1, &tmap_w, (kc + j) * kChunk, tile * kTileN, fb);
      }
      pdl_wait();
      for (long long i = 0; i < pre; ++i) {
        const long long u = u0 + i;
        const uint32_t fb = smem_u32(&full_bar[i]);
        const int kc = (int)(u % KC) * CPS;
        const uint32_t a = smem_u32(smem + i * STAGE);
#pragma unroll
        for (int j = 0; j < CPS; ++j) tma_load_2d(a + A_BYTES + j * B1, &tmap_x, (kc + j) * kChunk, 0, fb);
      }
      int i = (int)pre;
      for (long long u = u0 + pre; u < u1; ++u, ++i) {
        const int s = i % kStages;
        const uint32_t round = i / kStages;
        mbar_wait_bounded(smem_u32(&empty_bar[s]), (round & 1u) ^ 1u, abort_flag, p.status);
        const uint32_t fb = smem_u32(&full_bar[s]);
        mbar_arrive_expect_tx(fb, STAGE);
        if (!*abort_flag) {
          const int tile = (int)(u / KC), kc = (int)(u % KC) * CPS;
          const uint32_t a = smem_u32(smem + s * STAGE);
#pragma unroll
          for (int j = 0; j < CPS; ++j) tma_load_2d(a + j * A1, &tmap_w, (kc + j) * kChunk, tile * kTileN, fb);
#pragma unroll
          for (int j = 0; j < CPS; ++j) tma_load_2d(a + A_BYTES + j * B1, &tmap_x, (kc + j) * kChunk, 0, fb);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer: one segment (tile part) per accumulator, alternating buffers ----
    if (lane == 0) {
      int i = 0, seg = 0;
      long long u = u0;
      while (u < u1) {
        const long long tile_end = (u / KC + 1) * KC;
        const long long e = tile_end < u1 ? tile_end : u1;
        const int buf = seg & 1;
        mbar_wait_bounded(smem_u32(&tempty_bar[buf]), ((seg >> 1) & 1u) ^ 1u, abort_flag,
                          p.status);
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + buf * NB;
        for (long long v = u; v < e; ++v, ++i) {
          const int s = i % kStages;
          const uint32_t round = i / kStages;
          mbar_wait_bounded(smem_u32(&full_bar[s]), round & 1u, abort_flag, p.status);
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * STAGE);
#pragma unroll
          for (int j = 0; j < CPS; ++j) {
            const uint64_t da = smem_desc_sw128(a + j * A1);
            const uint64_t db = smem_desc_sw128(a + A_BYTES + j * B1);
#pragma unroll
            for (int kk = 0; kk < kChunk / 16; ++kk)   // K = 16 per MMA: +32 bytes in the row
              umma_bf16(tmem_d, da + 2 * kk, db + 2 * kk, IDESC,
                        (v > u || j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(smem_u32(&empty_bar[s]));       // stage free once these MMAs are done
        }
        umma_commit(smem_u32(&tfull_bar[buf]));       // this segment's accumulator is final
        u = e;
        ++seg;
      }
    }
    __syncwarp();
  } else {
    // ---- Epilogue: warps 2..5 own TMEM lane quarters (warp % 4) * 32 ----
    const int quarter = warp & 3;
    pdl_wait();   // global writes come after the predecessor grid (y / ws may alias its data)
    int seg = 0;
    long long u = u0;
    if (cl) {
      // Cluster split-K (NB = 64): the accumulator row of this thread stays in
      // registers until every CTA of the cluster is past its MMAs (first cluster
      // barrier below); then each value is pushed into the shared memory of the CTA
      // that sums that row.
      mbar_wait_bounded(smem_u32(&tfull_bar[0]), 0u, abort_flag, p.status);
      tc_fence_after();
      tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16), acc_lo);
      tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + 32u, acc_hi);
      u = u1;   // nothing left for the stream-K loop
    }
    while (u < u1) {
      const int tile = (int)(u / KC);
      const long long tile_end = (long long)(tile + 1) * KC;
      const long long e = tile_end < u1 ? tile_end : u1;
      const bool whole = (u == (long long)tile * KC) && (e == tile_end);
      const int buf = seg & 1;
      mbar_wait_bounded(smem_u32(&tfull_bar[buf]), (seg >> 1) & 1u, abort_flag, p.status);
      tc_fence_after();
      const int row = quarter * 32 + lane;                  // row of the tile
      const int m = tile * kTileN + row;                     // output feature of this thread
      const bool ok = !*abort_flag;
      const long long first_u = (long long)tile * KC;
      const int c_first = whole ? 0 : sk_owner(first_u, W, G);
      const int slot = whole ? 0 : (int)blockIdx.x - c_first;
      float* __restrict__ my_slot =
          p.ws + (((size_t)tile * p.max_seg + slot) * NB) * kTileN + row;
      // 32 accumulator columns (batch rows) at a time: read TMEM, then store bf16 (whole
      // tile) or this CTA's fp32 partial into its slot (tile shared by several CTAs).
#pragma unroll 1
      for (int c0 = 0; c0 < NB; c0 += 32) {
        float t[32];
        tmem_ld32(tmem_base + buf * NB + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c0, t);
        if (ok) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int b = c0 + j;
            if (b < p.Mb) {
              if (whole)
                p.y[(size_t)b * p.N + m] = __float2bfloat16_rn(t[j]);
              else
                my_slot[(size_t)b * kTileN] = t[j];
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[buf]));   // accumulator may be reused
      if (!whole) {
        // The last CTA to finish its part of this tile sums all parts, writes y and
        // resets the tile's counter for the next call.
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const int nseg = sk_owner(tile_end - 1, W, G) - c_first + 1;
        if (warp == 2 && lane == 0) {
          const int old = atomicAdd(&p.counters[tile], 1);
          *last_flag = (old == nseg - 1);
          if (old == nseg - 1) p.counters[tile] = 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last_flag) {
          __threadfence();
          const float* __restrict__ base = p.ws + ((size_t)tile * p.max_seg * NB) * kTileN + row;
#pragma unroll 1
          for (int b0 = 0; b0 < NB && b0 < p.Mb; b0 += 32) {
            float t[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) t[j] = 0.f;
            // Up to 4 parts' loads in flight together: one L2 round trip per 4 parts.
            for (int s0 = 0; s0 < nseg; s0 += 4) {
              float v[4][32];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const float* src = base + ((size_t)(s0 + q) * NB + b0) * kTileN;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  v[q][j] = (s0 + q < nseg && b0 + j < p.Mb) ? __ldcg(src + (size_t)j * kTileN) : 0.f;
              }
#pragma unroll
              for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int j = 0; j < 32; ++j) t[j] += v[q][j];
            }
            if (ok) {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (b0 + j < p.Mb) p.y[(size_t)(b0 + j) * p.N + m] = __float2bfloat16_rn(t[j]);
            }
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      u = e;
      ++seg;
    }
  }
  __syncwarp();
  if (cl) {
    // CTA rank q sums rows [q*128/S, (q+1)*128/S) of the tile.  Its receive buffer
    // (the idle ring) holds [S source ranks][64 columns][LR rows]; stores from the
    // peers are fire-and-forget, the second barrier makes them visible, and the sum
    // then reads local shared memory only.
    const int S = p.cluster;                 // 2, 4 or 8: every CTA sums 128 / S rows
    const int LR = kTileN / S;
    const uint32_t buf = smem_u32(smem);
    cluster_sync_all();   // every CTA's MMAs are done: its ring may be overwritten
    if (warp >= 2) {
      const int row = (warp & 3) * 32 + lane;
      const int q = row / LR;                        // owner of this row
      const int lr = row - q * LR;
      const uint32_t dst = dsmem_addr(buf, (uint32_t)q) +
                           (uint32_t)((crank * NB) * LR + lr) * 4u;
#pragma unroll
      for (int c = 0; c < 32; ++c) st_dsmem_f32(dst + (uint32_t)(c * LR) * 4u, acc_lo[c]);
#pragma unroll
      for (int c = 0; c < 32; ++c) st_dsmem_f32(dst + (uint32_t)((32 + c) * LR) * 4u, acc_hi[c]);
    }
    cluster_sync_all();   // all pushes have landed
    if (!*abort_flag) {
      // All six warps: item = (batch row b, 4 consecutive rows of this CTA's share),
      // S float4 reads of local shared memory and one 8-byte bf16x4 store.
      const int tile = (int)(blockIdx.x / S);
      const float* rb = reinterpret_cast<const float*>(smem);
      __nv_bfloat16* ybase = p.y + tile * kTileN + crank * LR;
      const int g4 = LR / 4, items = g4 * p.Mb;
      for (int it = threadIdx.x; it < items; it += kThreads) {
        const int b = it / g4, lr = (it - b * g4) * 4;
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < S; ++q) {
          const float4 v = *reinterpret_cast<const float4*>(rb + (q * NB + b) * LR + lr);
          a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
        }
        const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y);
        const __nv_bfloat162 hi = __floats2bfloat162_rn(a.z, a.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&lo);
        pk.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(ybase + (size_t)b * p.N + lr) = pk;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"((uint32_t)(2 * NB))
                 : "memory");
}

}  // namespace gemm

typedef CUresult (*EncodeTiledFn2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn2 encode_fn() {
  static EncodeTiledFn2 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn2>(ptr);
  }
  return fn;
}

// Row-major [rows, cols] bf16 matrix, box {64 cols, box_rows}, 128-byte swizzle.
static bool encode_rows(CUtensorMap* map, const void* base, long long rows, long long cols,
                        int box_rows, std::string* err) {
  EncodeTiledFn2 fn = encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is not available";
    return false;
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
    return false;
  }
  return true;
}

// Largest number of CTAs sharing one tile under the stream-K split of tiles * kc
// units over G CTAs (host mirror of the kernel's partition).
static int gemm_max_segments(int tiles, int kc, int G) {
  const long long W = (long long)tiles * kc;
  auto start = [&](long long c) { return c * W / G; };
  auto owner = [&](long long u) {
    long long c = u * G / W;
    while (c + 1 < G && start(c + 1) <= u) ++c;
    while (c > 0 && start(c) > u) --c;
    return c;
  };
  int mx = 1;
  for (int t = 0; t < tiles; ++t) {
    const int n = (int)(owner((long long)(t + 1) * kc - 1) - owner((long long)t * kc) + 1);
    if (n > mx) mx = n;
  }
  return mx;
}

template <int NB, int CPS>
static cudaError_t launch_gemm_nb(const void* x, const void* w, void* y, float* ws,
                                  size_t ws_floats, int32_t* counters, int Mb, int N, int K,
                                  int32_t* status, std::string* err, cudaStream_t stream) {
  CUtensorMap mw, mx;
  if (!encode_rows(&mw, w, N, K, gemm::kTileN, err) || !encode_rows(&mx, x, Mb, K, NB, err))
    return cudaErrorInvalidValue;
  constexpr size_t STAGE = gemm::Ring<NB, CPS>::kStageBytes;
  constexpr int S = gemm::Ring<NB, CPS>::kStages;
  const size_t smem = 1024 + S * STAGE + (2 * S + 4) * 8 + 16;
  auto kern = gemm::decode_gemm_kernel<NB, CPS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  gemm::Params p;
  p.y = reinterpret_cast<__nv_bfloat16*>(y);
  p.ws = ws;
  p.counters = counters;
  p.status = status;
  p.Mb = Mb; p.N = N; p.K = K;
  const int tiles = N / gemm::kTileN, kc = K / (gemm::kChunk * CPS);
  p.units = (long long)tiles * kc;
  // Cluster split-K when the tiles leave most SMs idle: csz CTAs per tile, csz <= 8, as
  // many as fit the SMs and the co-resident cluster count.
  int csz = NB == 64 ? sms / tiles : 1;   // the cluster path keeps a 64-column row in registers
  if (csz > 8) csz = 8;
  if (csz > kc) csz = kc;
  csz = csz >= 8 ? 8 : (csz >= 4 ? 4 : (csz >= 2 ? 2 : 1));   // a power of two dividing 128
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(gemm::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  while (csz >= 2) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = csz;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3(tiles * csz);
    cfg.numAttrs = 2;
    int nclusters = 0;
    if (cudaOccupancyMaxActiveClusters(&nclusters, kern, &cfg) == cudaSuccess &&
        nclusters >= tiles)
      break;
    cudaGetLastError();
    csz /= 2;
  }
  if (csz >= 2) {
    p.cluster = csz;
    p.max_seg = 1;
  } else {
    p.cluster = 0;
    cfg.numAttrs = 1;
    const int grid = (int)(p.units < sms ? p.units : sms);
    cfg.gridDim = dim3(grid);
    p.max_seg = gemm_max_segments(tiles, kc, grid);
    if ((size_t)tiles * p.max_seg * NB * gemm::kTileN > ws_floats) {
      *err = "decode GEMM workspace too small";
      return cudaErrorInvalidValue;
    }
  }
  e = cudaLaunchKernelEx(&cfg, kern, mw, mx, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

size_t decode_gemm_workspace_floats(int Mb, int N, int K) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int NB = Mb <= 64 ? 64 : (Mb <= 128 ? 128 : 256);
  const int tiles = N / gemm::kTileN;
  size_t mx = 0;
  for (int cps = 1; cps <= 4; cps *= 2) {     // the largest over the stage widths in use
    if ((K / 64) % cps) continue;
    const long long units = (long long)tiles * (K / (64 * cps));
    const int grid = (int)(units < sms ? units : sms);
    const size_t f = (size_t)tiles * gemm_max_segments(tiles, K / (64 * cps), grid) * NB * 128;
    if (f > mx) mx = f;
  }
  return mx;
}

cudaError_t launch_decode_gemm(const void* x, const void* w, void* y, float* ws, size_t ws_floats,
                               int32_t* counters, int Mb, int N, int K, int32_t* status,
                               std::string* err, cudaStream_t stream) {
  int cps = 4;                       // 4 consecutive 64-wide k-chunks per stage when K allows
  while (cps > 1 && (K / 64) % cps) cps /= 2;
#define LLMC_NB(NB)                                                                           \
  do {                                                                                        \
    if (cps >= 4) return launch_gemm_nb<NB, 4>(x, w, y, ws, ws_floats, counters, Mb, N, K, status, err, stream); \
    if (cps == 2) return launch_gemm_nb<NB, 2>(x, w, y, ws, ws_floats, counters, Mb, N, K, status, err, stream); \
    return launch_gemm_nb<NB, 1>(x, w, y, ws, ws_floats, counters, Mb, N, K, status, err, stream); \
  } while (0)
  if (Mb <= 64) LLMC_NB(64);
  if (Mb <= 128) LLMC_NB(128);
  LLMC_NB(256);
#undef LLMC_NB
}

}  // namespace llmc
