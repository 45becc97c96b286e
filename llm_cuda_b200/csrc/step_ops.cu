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

template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* __restrict__ gu, T* __restrict__ out,
                                                     int inter, long long total) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / inter;
    const int c = (int)(i - row * inter);
    const float g = to_f32(gu[row * 2 * inter + c]);
    const float u = to_f32(gu[row * 2 * inter + inter + c]);
    out[i] = from_f32<T>(g / (1.f + expf(-g)) * u);
  }
}

cudaError_t launch_add_rmsnorm(void* x, const void* delta, const void* w, void* h, int rows,
                               int hidden, float eps, int dtype, cudaStream_t stream) {
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

cudaError_t launch_swiglu(const void* gu, void* out, int rows, int inter, int dtype,
                          cudaStream_t stream) {
  const long long total = (long long)rows * inter;
  const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
  if (dtype == LLMC_F32)
    swiglu_kernel<float><<<grid, 256, 0, stream>>>((const float*)gu, (float*)out, inter, total);
  else if (dtype == LLMC_F16)
    swiglu_kernel<__half><<<grid, 256, 0, stream>>>((const __half*)gu, (__half*)out, inter, total);
  else
    swiglu_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>((const __nv_bfloat16*)gu,
                                                           (__nv_bfloat16*)out, inter, total);
  return cudaGetLastError();
}

}  // namespace llmc
