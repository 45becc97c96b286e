// One-shot all-reduce over NVLink peer memory fused with the residual add and RMSNorm
// of the decode step: for each row b,
//   s = sum over ranks of partial_r[b]   (fp32, rank order, rounded to the dtype)
//   x[b] = x[b] + s                      (the residual stream keeps the dtype)
//   h[b] = x[b] * rsqrt(mean(x[b]^2) + eps) * w
// replacing the NCCL all-reduce after o_proj / down_proj (the in-process sum of
// row-parallel partials at src/llm_cuda/parallel/tensor_parallel.py:83-90 of llm-cuda)
// and the add + RMSNorm that follows it (model.py:37-42, norm.py:31-33).
//
// Transport (no NCCL, no multicast): every rank owns, in memory mapped by all peers
// through CUDA IPC,
//   recv  [2][world][rows_cap][hidden]  partial rows pushed by each rank (double buffer)
//   flags [2][world][rows_cap] int32    epoch at which rank q's row b landed
// and keeps a private epoch counter per row.  CTA b of a call with epoch e:
//   1. pushes its partial row b into recv[e & 1][rank][b] of every rank (P2P stores),
//   2. fences at system scope and stores e into flags[e & 1][rank][b] of every rank,
//   3. waits (bounded by %globaltimer) until flags[e & 1][q][b] == e for every q,
//   4. sums the rows from its own recv (L2 reads), adds x and normalises.
// A rank reaches epoch e + 2 (which reuses slot e & 1) only after every peer has
// signalled e + 1, i.e. after every peer has finished reading slot e & 1 of call e.
#include <string>

#include "common.cuh"

namespace llmc {
namespace ar {

constexpr int kMaxWorld = 8;

struct Params {
  const void* partial;            // local [rows, hidden] (this rank's row-parallel output)
  void* const* recv;              // [world] device pointers to each rank's recv base
  int32_t* const* flags;          // [world] device pointers to each rank's flags base
  int32_t* epoch;                 // local [rows_cap]
  void* x;                        // [rows, hidden] residual, updated in place
  const void* w;                  // [hidden]
  void* h;                        // [rows, hidden] normalised output
  int32_t* status;
  int rank, world, rows, rows_cap, hidden;
  float eps;
};

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One CTA per row; each thread owns NV 16-byte vectors of the row.
template <typename T, int NV>
__global__ void __launch_bounds__(1024) allreduce_add_rmsnorm_kernel(const Params p) {
  constexpr int VEC = 16 / sizeof(T);
  const int b = blockIdx.x;
  const int nvec = p.hidden / VEC;
  __shared__ int32_t s_epoch;
  __shared__ int s_fail;
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();   // the partial and x come from the previous kernels

  if (threadIdx.x == 0) {
    s_epoch = p.epoch[b] + 1;
    s_fail = 0;
  }
  __syncthreads();
  const int32_t e = s_epoch;
  const int par = e & 1;
  const size_t row_elems = (size_t)p.hidden;
  const size_t slot_stride = (size_t)p.world * p.rows_cap * row_elems;   // elements per parity

  // 1. push this rank's row b to every rank (itself included)
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.partial) +
                                                    (size_t)b * row_elems);
  uint4 mine[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) mine[k] = __ldcg(src + i);
  }
  const size_t dst_off = (size_t)par * slot_stride +
                         ((size_t)p.rank * p.rows_cap + b) * row_elems;
  for (int q = 0; q < p.world; ++q) {
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.recv[q]) + dst_off);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) dst[i] = mine[k];
    }
  }
  // 2. make the pushes visible system-wide, then publish the epoch on every rank
  __threadfence_system();
  __syncthreads();
  const size_t flag_off = (size_t)par * p.world * p.rows_cap + (size_t)p.rank * p.rows_cap + b;
  if (threadIdx.x < p.world) st_release_sys(p.flags[threadIdx.x] + flag_off, e);
  // 3. wait (bounded) for every rank's row b of this epoch
  if (threadIdx.x < p.world) {
    const int32_t* f = p.flags[p.rank] + (size_t)par * p.world * p.rows_cap +
                       (size_t)threadIdx.x * p.rows_cap + b;
    const unsigned long long t0 = globaltimer_ns();
    unsigned it = 0;
    while (ld_acquire_sys(f) != e) {
      if ((++it & 255u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicOr(p.status, kStatusWaitTimeout);
        s_fail = 1;
        break;
      }
    }
  }
  __syncthreads();
  if (s_fail) {
    // Rows stay as they were and the status word reports the timeout.  The epoch still
    // advances: this rank has already published e to its peers, so reusing e on the
    // next call would pass the wait on the peers' stale flags of this call.
    if (threadIdx.x == 0) p.epoch[b] = e;
    return;
  }
  // 4. sum in rank order from this rank's recv slot, add the residual, normalise
  const T* rv = reinterpret_cast<const T*>(p.recv[p.rank]) + (size_t)par * slot_stride +
                (size_t)b * row_elems;
  T* xr = reinterpret_cast<T*>(p.x) + (size_t)b * row_elems;
  float xs[NV][VEC];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    float acc[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] = 0.f;
    for (int q = 0; q < p.world; ++q) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(rv + (size_t)q * p.rows_cap * row_elems) + i);
      const T* ve = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] += to_f32(ve[j]);
    }
    uint4 xv = reinterpret_cast<const uint4*>(xr)[i];
    T* xe = reinterpret_cast<T*>(&xv);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      // all-reduce result in the dtype, then the residual add in the dtype
      xe[j] = from_f32<T>(to_f32(xe[j]) + to_f32(from_f32<T>(acc[j])));
      xs[k][j] = to_f32(xe[j]);
      ss = fmaf(xs[k][j], xs[k][j], ss);
    }
    reinterpret_cast<uint4*>(xr)[i] = xv;
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / p.hidden + p.eps);
  const uint4* wv = reinterpret_cast<const uint4*>(p.w);
  uint4* hr = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.h) + (size_t)b * row_elems);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    const uint4 ww = __ldg(wv + i);
    const T* we = reinterpret_cast<const T*>(&ww);
    uint4 ov;
    T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int j = 0; j < VEC; ++j) oe[j] = from_f32<T>(xs[k][j] * r * to_f32(we[j]));
    hr[i] = ov;
  }
  if (threadIdx.x == 0) p.epoch[b] = e;
}

}  // namespace ar

// Sizes of one rank's shared region: recv (elements of the dtype), flags (int32).
size_t ar_recv_bytes(int world, int rows_cap, int hidden, int elem) {
  return (size_t)2 * world * rows_cap * hidden * elem;
}
size_t ar_flag_bytes(int world, int rows_cap) { return (size_t)2 * world * rows_cap * 4; }

cudaError_t launch_allreduce_add_rmsnorm(const ar::Params& p, int dtype, std::string* err,
                                         cudaStream_t stream) {
  const int elem = dtype == LLMC_F32 ? 4 : 2;
  const int vec = 16 / elem;
  if (p.hidden % vec) {
    *err = "hidden must be a multiple of 16 bytes";
    return cudaErrorInvalidValue;
  }
  const int nvec = p.hidden / vec;
  int threads = ((nvec + 31) / 32) * 32;
  if (threads < 64) threads = 64;
  if (threads > 1024) threads = 1024;
  const int nv = (nvec + threads - 1) / threads;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.rows);
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
#define LLMC_AR(TT, NV) cudaLaunchKernelEx(&cfg, ar::allreduce_add_rmsnorm_kernel<TT, NV>, p)
#define LLMC_AR_T(TT)                                          \
  do {                                                         \
    if (nv == 1) e = LLMC_AR(TT, 1);                           \
    else if (nv == 2) e = LLMC_AR(TT, 2);                      \
    else if (nv <= 4) e = LLMC_AR(TT, 4);                      \
    else { *err = "hidden too large"; return cudaErrorInvalidValue; } \
  } while (0)
  cudaError_t e;
  if (dtype == LLMC_F32) LLMC_AR_T(float);
  else if (dtype == LLMC_F16) LLMC_AR_T(__half);
  else LLMC_AR_T(__nv_bfloat16);
#undef LLMC_AR_T
#undef LLMC_AR
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace llmc
