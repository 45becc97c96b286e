// Fused element-wise kernels of the decode step around the attention path.
//
//  * add_rmsnorm: x += delta (the residual add, model.py:37,42 of llm-cuda), then
//    h = x * rsqrt(mean(x^2) + eps) * w (RMSNorm, norm.py:31-33).  One CTA per row;
//    the sum of squares is accumulated in fp32 and each output is rounded once.
//  * swiglu: out = silu(gate) * up with gate/up the two halves of the fused
//    gate_up projection (kernels/triton/swiglu.py:103-107), fp32 math, one rounding.
// They replace 6-8 tiny PyTorch kernels per layer in the config-5 decode step.
#include "common.cuh"

namespace llmc {

template <typename T>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(T* __restrict__ x,
                                                          const T* __restrict__ delta,
                                                          const T* __restrict__ w,
                                                          T* __restrict__ h, int hidden,
                                                          float eps) {
  pdl_launch_dependents();
  pdl_wait();
  const size_t row = blockIdx.x;
  T* xr = x + row * hidden;
  const T* dr = delta ? delta + row * hidden : nullptr;
  T* hr = h + row * hidden;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float v = to_f32(xr[i]);
    if (dr) {
      v = to_f32(from_f32<T>(v + to_f32(dr[i])));   // the residual stream keeps the dtype
      xr[i] = from_f32<T>(v);
    }
    ss = fmaf(v, v, ss);
  }
  __shared__ float red[32];
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    hr[i] = from_f32<T>(to_f32(xr[i]) * r * to_f32(w[i]));
}

// The same with 16-byte vectors held in registers: each thread loads NV vectors of
// x (and delta) once, the row's sum of squares is reduced across the CTA, and the
// normalised output is written from registers.  Every load is issued before the
// first reduction, so a row costs about one memory round trip.
template <typename T, int NV>
__global__ void __launch_bounds__(1024) add_rmsnorm_vec_kernel(T* __restrict__ x,
                                                               const T* __restrict__ delta,
                                                               const T* __restrict__ w,
                                                               T* __restrict__ h, int hidden,
                                                               float eps) {
  constexpr int VEC = 16 / sizeof(T);
  pdl_launch_dependents();
  pdl_wait();   // x / delta come from the previous kernel
  const size_t row = blockIdx.x;
  const int nvec = hidden / VEC;
  uint4* xr = reinterpret_cast<uint4*>(x + row * hidden);
  const uint4* dr = delta ? reinterpret_cast<const uint4*>(delta + row * hidden) : nullptr;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* hr = reinterpret_cast<uint4*>(h + row * hidden);
  uint4 xv[NV], dv[NV];
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < nvec) {
      xv[k] = xr[i];
      if (dr) dv[k] = __ldg(dr + i);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    T* xe = reinterpret_cast<T*>(&xv[k]);
    if (dr) {
      const T* de = reinterpret_cast<const T*>(&dv[k]);
#pragma unroll
      for (int e = 0; e < VEC; ++e) xe[e] = from_f32<T>(to_f32(xe[e]) + to_f32(de[e]));
      xr[i] = xv[k];                                  // the residual stream keeps the dtype
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) ss = fmaf(to_f32(xe[e]), to_f32(xe[e]), ss);
  }
  __shared__ float red[32];
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / hidden + eps);
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i >= nvec) continue;
    const uint4 wv = __ldg(wr + i);
    const T* xe = reinterpret_cast<const T*>(&xv[k]);
    const T* we = reinterpret_cast<const T*>(&wv);
    uint4 ov;
    T* oe = reinterpret_cast<T*>(&ov);
#pragma unroll
    for (int e = 0; e < VEC; ++e) oe[e] = from_f32<T>(to_f32(xe[e]) * r * to_f32(we[e]));
    hr[i] = ov;
  }
}

// Row-wise argmax (first index of the maximum; NaN counts as the maximum, as in
// torch.argmax), replacing the greedy pick of the decode loop (model.py:214).  A row is
// cut into `gridDim.x` chunks; each CTA folds its chunk into a 64-bit key
// (order-preserving value bits << 32 | ~index) with atomicMax, and the CTA that
// completes the row writes the index and re-arms the key and the counter.
__device__ __forceinline__ unsigned long long argmax_key(float f, unsigned idx) {
  unsigned u = __float_as_uint(f);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (0xFFFFFFFFu - idx);
}

template <typename T>
__global__ void __launch_bounds__(256) argmax_rows_kernel(const T* __restrict__ x,
                                                          int64_t* __restrict__ out, int n,
                                                          unsigned long long* keys,
                                                          int* counters) {
  const int row = blockIdx.y;
  const int per = (n + gridDim.x - 1) / gridDim.x;
  const int lo = blockIdx.x * per, hi = min(n, lo + per);
  const T* xr = x + (size_t)row * n;
  unsigned long long best = 0;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const unsigned long long k = argmax_key(to_f32(__ldg(xr + i)), (unsigned)i);
    best = k > best ? k : best;
  }
  for (int o = 16; o; o >>= 1) {
    const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
    best = v > best ? v : best;
  }
  __shared__ unsigned long long red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = red[w] > best ? red[w] : best;
    atomicMax(keys + row, best);
    __threadfence();
    if (atomicAdd(counters + row, 1) == (int)gridDim.x - 1) {
      __threadfence();
      const unsigned long long k = atomicExch(keys + row, 0ull);
      out[row] = (int64_t)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull));
      counters[row] = 0;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* __restrict__ gu, T* __restrict__ out,
                                                     int inter, long long total) {
  pdl_launch_dependents();
  pdl_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / inter;
    const int c = (int)(i - row * inter);
    const float g = to_f32(gu[row * 2 * inter + c]);
    const float u = to_f32(gu[row * 2 * inter + inter + c]);
    out[i] = from_f32<T>(g / (1.f + expf(-g)) * u);
  }
}

// Launch with programmatic stream serialization: the kernel's prologue may overlap
// the previous kernel, whose results it reads only after griddepcontrol.wait.
template <typename... KArgs, typename... Args>
static void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t stream,
                       Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

template <typename T>
static bool launch_add_rmsnorm_vec(void* x, const void* delta, const void* w, void* h, int rows,
                                   int hidden, float eps, cudaStream_t stream) {
  constexpr int VEC = 16 / sizeof(T);
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (hidden % VEC || !al(x) || !al(w) || !al(h) || (delta && !al(delta))) return false;
  const int nvec = hidden / VEC;
  int threads = ((nvec + 31) / 32) * 32;
  if (threads > 1024) threads = 1024;
  const int nv = (nvec + threads - 1) / threads;
#define LLMC_RMS(NV)                                                                         \
  launch_pdl(add_rmsnorm_vec_kernel<T, NV>, dim3(rows), dim3(threads), stream, (T*)x,       \
             (const T*)delta, (const T*)w, (T*)h, hidden, eps)
  if (nv == 1) LLMC_RMS(1);
  else if (nv == 2) LLMC_RMS(2);
  else if (nv <= 4) LLMC_RMS(4);
  else if (nv <= 8) LLMC_RMS(8);
  else return false;
#undef LLMC_RMS
  return true;
}

cudaError_t launch_add_rmsnorm(void* x, const void* delta, const void* w, void* h, int rows,
                               int hidden, float eps, int dtype, cudaStream_t stream) {
  bool done = false;
  if (dtype == LLMC_F32) done = launch_add_rmsnorm_vec<float>(x, delta, w, h, rows, hidden, eps, stream);
  else if (dtype == LLMC_F16) done = launch_add_rmsnorm_vec<__half>(x, delta, w, h, rows, hidden, eps, stream);
  else done = launch_add_rmsnorm_vec<__nv_bfloat16>(x, delta, w, h, rows, hidden, eps, stream);
  if (done) return cudaGetLastError();
  if (dtype == LLMC_F32)
    add_rmsnorm_kernel<float><<<rows, 256, 0, stream>>>((float*)x, (const float*)delta,
                                                        (const float*)w, (float*)h, hidden, eps);
  else if (dtype == LLMC_F16)
    add_rmsnorm_kernel<__half><<<rows, 256, 0, stream>>>((__half*)x, (const __half*)delta,
                                                         (const __half*)w, (__half*)h, hidden, eps);
  else
    add_rmsnorm_kernel<__nv_bfloat16><<<rows, 256, 0, stream>>>(
        (__nv_bfloat16*)x, (const __nv_bfloat16*)delta, (const __nv_bfloat16*)w,
        (__nv_bfloat16*)h, hidden, eps);
  return cudaGetLastError();
}

// 16-byte vectors: thread i handles elements [VEC*i, VEC*i + VEC) of the [rows, inter]
// output (inter % VEC == 0, so a vector never crosses a row).
template <typename T>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(const T* __restrict__ gu,
                                                         T* __restrict__ out, int inter,
                                                         long long nvec) {
  constexpr int VEC = 16 / sizeof(T);
  pdl_launch_dependents();
  pdl_wait();
  const int vpr = inter / VEC;   // vectors per row
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nvec;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vpr;
    const int cv = (int)(i - row * vpr);
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(gu + row * 2 * inter) + cv);
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(gu + row * 2 * inter + inter) + cv);
    const T* ge = reinterpret_cast<const T*>(&g);
    const T* ue = reinterpret_cast<const T*>(&u);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float gv = to_f32(ge[e]);
      oe[e] = from_f32<T>(gv / (1.f + expf(-gv)) * to_f32(ue[e]));
    }
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

template <typename T>
static bool launch_swiglu_vec(const void* gu, void* out, int rows, int inter,
                              cudaStream_t stream) {
  constexpr int VEC = 16 / sizeof(T);
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (inter % VEC || !al(gu) || !al(out)) return false;
  const long long nvec = (long long)rows * inter / VEC;
  const int grid = (int)((nvec + 255) / 256 < 148 * 8 ? (nvec + 255) / 256 : 148 * 8);
  launch_pdl(swiglu_vec_kernel<T>, dim3(grid), dim3(256), stream, (const T*)gu, (T*)out, inter,
             nvec);
  return true;
}

cudaError_t launch_swiglu(const void* gu, void* out, int rows, int inter, int dtype,
                          cudaStream_t stream) {
  bool done;
  if (dtype == LLMC_F32) done = launch_swiglu_vec<float>(gu, out, rows, inter, stream);
  else if (dtype == LLMC_F16) done = launch_swiglu_vec<__half>(gu, out, rows, inter, stream);
  else done = launch_swiglu_vec<__nv_bfloat16>(gu, out, rows, inter, stream);
  if (done) return cudaGetLastError();
  const long long total = (long long)rows * inter;
  const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
  if (dtype == LLMC_F32)
    launch_pdl(swiglu_kernel<float>, dim3(grid), dim3(256), stream, (const float*)gu, (float*)out,
               inter, total);
  else if (dtype == LLMC_F16)
    launch_pdl(swiglu_kernel<__half>, dim3(grid), dim3(256), stream, (const __half*)gu,
               (__half*)out, inter, total);
  else
    launch_pdl(swiglu_kernel<__nv_bfloat16>, dim3(grid), dim3(256), stream,
               (const __nv_bfloat16*)gu, (__nv_bfloat16*)out, inter, total);
  return cudaGetLastError();
}

cudaError_t launch_argmax(const void* x, int64_t* out, int rows, int n, int dtype,
                          unsigned long long* keys, int* counters, int sms, cudaStream_t stream) {
  int splits = (n + 4095) / 4096;
  const int want = (4 * sms + rows - 1) / rows;
  if (splits > want) splits = want;
  if (splits < 1) splits = 1;
  dim3 grid(splits, rows);
  if (dtype == LLMC_F32)
    argmax_rows_kernel<float><<<grid, 256, 0, stream>>>((const float*)x, out, n, keys, counters);
  else if (dtype == LLMC_F16)
    argmax_rows_kernel<__half><<<grid, 256, 0, stream>>>((const __half*)x, out, n, keys, counters);
  else
    argmax_rows_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>((const __nv_bfloat16*)x, out, n,
                                                                 keys, counters);
  return cudaGetLastError();
}

}  // namespace llmc
