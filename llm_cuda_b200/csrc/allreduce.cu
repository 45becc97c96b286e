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
//   recv [2][world][rows_cap][hidden * elem / 4]  8-byte words {4 data bytes, epoch}
// and keeps a private epoch counter per row.  CTA b of a call with epoch e:
//   1. pushes its partial row b into recv[e & 1][rank][b] of every peer with 8-byte
//      stores, each carrying 4 bytes of the row and the epoch e,
//   2. polls (bounded by %globaltimer) its own recv[e & 1][q][b] of every peer q until
//      every word carries e: an aligned 8-byte store is seen whole or not at all, so a
//      word with epoch e holds this call's data, and no fence or separate flag (with
//      its extra NVLink round trip) is needed,
//   3. sums the rows in rank order (its own from registers), adds x and normalises.
// Words from older calls carry older epochs, so nothing is ever cleared.  A rank
// reaches epoch e + 2 (which reuses slot e & 1) only after every peer has sent its
// e + 1 words, i.e. after every peer has finished call e (each call waits for the
// previous kernel before it pushes).
#include <cstdlib>
#include <cstring>
#include <string>

#include "common.cuh"

namespace llmc {
namespace ar {

struct Params {
  const void* partial;            // local [rows, hidden] (this rank's row-parallel output)
  void* const* recv;              // [world] device pointers to each rank's recv base
  int32_t* const* flags;          // unused (the words carry their epoch)
  int32_t* epoch;                 // local [rows_cap]
  void* x;                        // [rows, hidden] residual, updated in place
  const void* w;                  // [hidden]
  void* h;                        // [rows, hidden] normalised output
  int32_t* status;
  int rank, world, rows, rows_cap, hidden;
  float eps;
};

__device__ __forceinline__ void st_ll(uint64_t* p, uint32_t data, uint32_t flag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(data), "r"(flag)
               : "memory");
}
__device__ __forceinline__ void ld_ll(const uint64_t* p, uint32_t& data, uint32_t& flag) {
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(data), "=r"(flag) : "l"(p)
               : "memory");
}

// One CTA per row; each thread owns NV 16-byte vectors of the row (4 words each).
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
    // After a timeout the ranks' epochs may be out of step: later calls (e.g. replays
    // of a captured graph) fail at once instead of each waiting out the deadline.
    s_fail = (*reinterpret_cast<volatile int32_t*>(p.status) & kStatusWaitTimeout) ? 1 : 0;
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) p.epoch[b] = s_epoch;
    return;
  }
  const uint32_t e = (uint32_t)s_epoch;
  const int par = e & 1;
  const size_t row_words = (size_t)nvec * 4;                       // 8-byte words per row
  const size_t slot_words = (size_t)p.world * p.rows_cap * row_words;

  // 1. push this rank's row b to every peer (its own copy stays in registers)
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.partial) +
                                                    (size_t)b * p.hidden);
  uint4 mine[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) mine[k] = __ldcg(src + i);
  }
  const size_t my_row = (size_t)par * slot_words + ((size_t)p.rank * p.rows_cap + b) * row_words;
  for (int q = 0; q < p.world; ++q) {
    if (q == p.rank) continue;
    uint64_t* dst = reinterpret_cast<uint64_t*>(p.recv[q]) + my_row;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i < nvec) {   // word j of vector i at j * nvec + i: each store is warp-contiguous
        st_ll(dst + 0 * nvec + i, mine[k].x, e);
        st_ll(dst + 1 * nvec + i, mine[k].y, e);
        st_ll(dst + 2 * nvec + i, mine[k].z, e);
        st_ll(dst + 3 * nvec + i, mine[k].w, e);
      }
    }
  }
  // 2 + 3. sum in rank order: own row from registers, each peer's words polled until
  // they carry this epoch (bounded wait), then the residual add and the norm
  const uint64_t* rv = reinterpret_cast<const uint64_t*>(p.recv[p.rank]) + (size_t)par * slot_words;
  T* xr = reinterpret_cast<T*>(p.x) + (size_t)b * p.hidden;
  float xs[NV][VEC];
  float ss = 0.f;
  bool fail = false;
  const unsigned long long t0 = globaltimer_ns();
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    float acc[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] = 0.f;
    for (int q = 0; q < p.world; ++q) {
      uint4 v;
      if (q == p.rank) {
        v = mine[k];
      } else {
        const uint64_t* w = rv + ((size_t)q * p.rows_cap + b) * row_words + i;
        uint32_t d[4], f[4];
        unsigned it = 0;
        for (;;) {
          ld_ll(w + 0 * nvec, d[0], f[0]);
          ld_ll(w + 1 * nvec, d[1], f[1]);
          ld_ll(w + 2 * nvec, d[2], f[2]);
          ld_ll(w + 3 * nvec, d[3], f[3]);
          if (f[0] == e && f[1] == e && f[2] == e && f[3] == e) break;
          if (fail || ((++it & 63u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs)) {
            fail = true;
            break;
          }
        }
        v = make_uint4(d[0], d[1], d[2], d[3]);
      }
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
  }
  if (fail) {
    atomicOr(p.status, kStatusWaitTimeout);
    s_fail = 1;
  }
  __syncthreads();
  if (s_fail) {
    // Rows stay as they were and the status word reports the timeout.  The epoch still
    // advances: this rank has already pushed e-words to its peers, so reusing e on the
    // next call could let a peer take this call's words for the next call's.
    if (threadIdx.x == 0) p.epoch[b] = (int32_t)e;
    return;
  }
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    uint4 xv;
    T* xe = reinterpret_cast<T*>(&xv);
#pragma unroll
    for (int j = 0; j < VEC; ++j) xe[j] = from_f32<T>(xs[k][j]);
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
  uint4* hr = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.h) + (size_t)b * p.hidden);
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
  if (threadIdx.x == 0) p.epoch[b] = (int32_t)e;
}

// Two-shot variant for larger groups: the one-shot push costs (world - 1) full rows per
// rank, this one 2 * (world - 1) / world of a row, at the price of a second hop.
//   1. reduce-scatter: rank r owns the vectors [r * nvs, (r + 1) * nvs) of every row
//      (nvs = vectors / world); every rank pushes each vector to its owner;
//   2. the owner sums its slice in rank order, adds the residual (x_new), and reduces
//      the slice's sum of squares;
//   3. all-gather: the owner pushes x_new of its slice and that sum to every rank;
//   4. every rank sums the slice sums in rank order (the same bits on every rank) and
//      normalises the full row.
// Region: RS area [2][world][rows_cap][4 * nvs] words, then AG area
// [2][world][rows_cap][4 * nvs + 1] words (the last word of an AG row is the slice's
// sum of squares).
template <typename T, int NV>
__global__ void __launch_bounds__(1024) allreduce_add_rmsnorm_2shot_kernel(const Params p) {
  constexpr int VEC = 16 / sizeof(T);
  const int b = blockIdx.x;
  const int nvec = p.hidden / VEC;
  const int nvs = nvec / p.world;                 // vectors per owner slice
  const size_t sw = (size_t)4 * nvs;              // words per slice
  __shared__ int32_t s_epoch;
  __shared__ int s_fail;
  __shared__ float red[32];
  __shared__ float s_part[8];
  pdl_launch_dependents();
  pdl_wait();   // the partial and x come from the previous kernels

  if (threadIdx.x == 0) {
    s_epoch = p.epoch[b] + 1;
    // After a timeout the ranks' epochs may be out of step: later calls (e.g. replays
    // of a captured graph) fail at once instead of each waiting out the deadline.
    s_fail = (*reinterpret_cast<volatile int32_t*>(p.status) & kStatusWaitTimeout) ? 1 : 0;
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) p.epoch[b] = s_epoch;
    return;
  }
  const uint32_t e = (uint32_t)s_epoch;
  const int par = e & 1;
  const size_t rs_par = (size_t)p.world * p.rows_cap * sw;           // RS words per parity
  const size_t ag_base = 2 * rs_par;
  const size_t ag_par = (size_t)p.world * p.rows_cap * (sw + 1);
  uint64_t* own = reinterpret_cast<uint64_t*>(p.recv[p.rank]);

  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.partial) +
                                                    (size_t)b * p.hidden);
  T* xr = reinterpret_cast<T*>(p.x) + (size_t)b * p.hidden;
  uint4 mine[NV];
  bool fail = false;
  const unsigned long long t0 = globaltimer_ns();
  auto poll4 = [&](const uint64_t* w, size_t stride, uint4& v) {
    uint32_t d[4], f[4];
    unsigned it = 0;
    for (;;) {
#pragma unroll
      for (int j = 0; j < 4; ++j) ld_ll(w + j * stride, d[j], f[j]);
      if (f[0] == e && f[1] == e && f[2] == e && f[3] == e) break;
      if (fail || ((++it & 63u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs)) {
        fail = true;
        break;
      }
    }
    v = make_uint4(d[0], d[1], d[2], d[3]);
  };
  // 1. reduce-scatter push: vector i goes to its owner i / nvs
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    mine[k] = __ldcg(src + i);
    const int q = i / nvs, li = i - q * nvs;
    if (q == p.rank) continue;
    uint64_t* dst = reinterpret_cast<uint64_t*>(p.recv[q]) + (size_t)par * rs_par +
                    ((size_t)p.rank * p.rows_cap + b) * sw + li;
    st_ll(dst + 0 * nvs, mine[k].x, e);
    st_ll(dst + 1 * nvs, mine[k].y, e);
    st_ll(dst + 2 * nvs, mine[k].z, e);
    st_ll(dst + 3 * nvs, mine[k].w, e);
  }
  // 2. the owned slice: sum in rank order, residual add, sum of squares
  float xs[NV][VEC];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec || i / nvs != p.rank) continue;
    const int li = i - p.rank * nvs;
    float acc[VEC];
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[j] = 0.f;
    for (int q = 0; q < p.world; ++q) {
      uint4 v;
      if (q == p.rank) v = mine[k];
      else poll4(own + (size_t)par * rs_par + ((size_t)q * p.rows_cap + b) * sw + li, nvs, v);
      const T* ve = reinterpret_cast<const T*>(&v);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[j] += to_f32(ve[j]);
    }
    const uint4 xv = reinterpret_cast<const uint4*>(xr)[i];
    const T* xe = reinterpret_cast<const T*>(&xv);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      xs[k][j] = to_f32(from_f32<T>(to_f32(xe[j]) + to_f32(from_f32<T>(acc[j]))));
      ss = fmaf(xs[k][j], xs[k][j], ss);
    }
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) s_part[p.rank] = t;
  }
  __syncthreads();
  // 3. all-gather push: x_new of the owned slice, then the slice's sum of squares
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec || i / nvs != p.rank) continue;
    const int li = i - p.rank * nvs;
    uint4 xv;
    T* xe = reinterpret_cast<T*>(&xv);
#pragma unroll
    for (int j = 0; j < VEC; ++j) xe[j] = from_f32<T>(xs[k][j]);
    mine[k] = xv;   // this rank's own x_new vector
    for (int q = 0; q < p.world; ++q) {
      if (q == p.rank) continue;
      uint64_t* dst = reinterpret_cast<uint64_t*>(p.recv[q]) + ag_base + (size_t)par * ag_par +
                      ((size_t)p.rank * p.rows_cap + b) * (sw + 1) + li;
      st_ll(dst + 0 * nvs, xv.x, e);
      st_ll(dst + 1 * nvs, xv.y, e);
      st_ll(dst + 2 * nvs, xv.z, e);
      st_ll(dst + 3 * nvs, xv.w, e);
    }
  }
  if (threadIdx.x < p.world && threadIdx.x != p.rank) {
    uint64_t* dst = reinterpret_cast<uint64_t*>(p.recv[threadIdx.x]) + ag_base +
                    (size_t)par * ag_par + ((size_t)p.rank * p.rows_cap + b) * (sw + 1) + sw;
    st_ll(dst, __float_as_uint(s_part[p.rank]), e);
  }
  // 4. the other slices and the slice sums
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    const int q = i / nvs, li = i - q * nvs;
    if (q == p.rank) continue;
    uint4 v;
    poll4(own + ag_base + (size_t)par * ag_par + ((size_t)q * p.rows_cap + b) * (sw + 1) + li,
          nvs, v);
    mine[k] = v;
    const T* ve = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int j = 0; j < VEC; ++j) xs[k][j] = to_f32(ve[j]);
  }
  if (threadIdx.x < p.world && threadIdx.x != p.rank) {
    const uint64_t* w = own + ag_base + (size_t)par * ag_par +
                        ((size_t)threadIdx.x * p.rows_cap + b) * (sw + 1) + sw;
    uint32_t d = 0, f = 0;
    unsigned it = 0;
    for (;;) {
      ld_ll(w, d, f);
      if (f == e) break;
      if (fail || ((++it & 63u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs)) {
        fail = true;
        break;
      }
    }
    s_part[threadIdx.x] = __uint_as_float(d);
  }
  if (fail) {
    atomicOr(p.status, kStatusWaitTimeout);
    s_fail = 1;
  }
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) p.epoch[b] = (int32_t)e;   // as in the one-shot kernel
    return;
  }
  float tot = 0.f;
  for (int q = 0; q < p.world; ++q) tot += s_part[q];   // rank order: the same on every rank
  const float r = rsqrtf(tot / p.hidden + p.eps);
  const uint4* wv = reinterpret_cast<const uint4*>(p.w);
  uint4* hr = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.h) + (size_t)b * p.hidden);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    reinterpret_cast<uint4*>(xr)[i] = mine[k];
    const uint4 ww = __ldg(wv + i);
    const T* we = reinterpret_cast<const T*>(&ww);
    uint4 ov;
    T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int j = 0; j < VEC; ++j) oe[j] = from_f32<T>(xs[k][j] * r * to_f32(we[j]));
    hr[i] = ov;
  }
  if (threadIdx.x == 0) p.epoch[b] = (int32_t)e;
}

}  // namespace ar

// Size of one rank's shared region: two parities of [world][rows_cap] rows of 8-byte
// words, each carrying 4 bytes of the row.  No flag region is needed.
// The region holds either layout: one-shot 2 * world * rows_cap * W words (W = words
// per row), two-shot 2 * rows_cap * W words of reduce-scatter slices plus
// 2 * world * rows_cap * (W / world + 1) words of all-gather slices with their sums.
size_t ar_recv_bytes(int world, int rows_cap, int hidden, int elem) {
  const size_t w = (size_t)hidden * elem / 4;
  const size_t one = (size_t)2 * world * rows_cap * w;
  const size_t two = (size_t)2 * rows_cap * w + (size_t)2 * world * rows_cap * (w / world + 1);
  return (one > two ? one : two) * 8;
}

// One-shot up to `kOneShotMaxWorld` ranks, two-shot above, unless LLMC_AR_ALGO names
// one ("one_shot" / "two_shot"; read once per process, for measurements).
constexpr int kOneShotMaxWorld = 2;
static int ar_algo_override() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("LLMC_AR_ALGO");
    v = (s && !strcmp(s, "one_shot")) ? 1 : (s && !strcmp(s, "two_shot")) ? 2 : 0;
  }
  return v;
}
size_t ar_flag_bytes(int, int) { return 0; }

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
  const int ov = ar_algo_override();
  const bool two = nvec % p.world == 0 && p.world > 1 &&
                   (ov == 2 || (ov == 0 && p.world > kOneShotMaxWorld));
#define LLMC_AR(TT, NV)                                                                      \
  (two ? cudaLaunchKernelEx(&cfg, ar::allreduce_add_rmsnorm_2shot_kernel<TT, NV>, p)        \
       : cudaLaunchKernelEx(&cfg, ar::allreduce_add_rmsnorm_kernel<TT, NV>, p))
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
