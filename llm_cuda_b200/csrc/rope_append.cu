// Fused RoPE on the new tokens + KV-page append.
//
// One CTA per sequence b.  The CTA reads the sequence's current length once,
// rotates q and k of its S new tokens, writes rotated k and raw v straight into
// the physical pages named by the block table, writes rotated q, and finally
// advances seq_lens[b] by S.  Only CTA b touches seq_lens[b], so the in-place
// update is race-free and the step needs no host bookkeeping (graph-capturable).
//
// Work unit = (token, head, 16-byte chunk).  For RoPE a unit pairs the chunk at
// element i of the first half with the chunk at i + d/2 (rotate_half partner),
// so each thread issues 16-byte loads and stores only.
//
// Rounding matches the reference's torch path (rotary.py:104-109): products
// x*cos and rotate_half(x)*sin are rounded to the storage dtype, then the sum.
// For fp32 the same three rounded operations are used (no FMA contraction).
#include "common.cuh"

namespace llmc {

template <typename T, int VEC>
__global__ void __launch_bounds__(512) rope_append_kernel(
    const T* __restrict__ q_in, const T* __restrict__ k_in, const T* __restrict__ v_in,
    T* __restrict__ q_out, T* __restrict__ k_pages, T* __restrict__ v_pages,
    const int32_t* __restrict__ block_table, int32_t* __restrict__ seq_lens,
    const T* __restrict__ cos_tab, const T* __restrict__ sin_tab, int S, int Hq, int Hkv, int d,
    int P, int max_pages, int num_pages, int rope_max_pos, int32_t* __restrict__ status) {
  using Vec = typename std::conditional<VEC * sizeof(T) == 16, uint4,
              typename std::conditional<VEC * sizeof(T) == 8, uint2, T>::type>::type;
  const int b = blockIdx.x;
  pdl_launch_dependents();   // the decode kernel may start its prologue now
  __shared__ int s_pos0;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const int pos0 = seq_lens[b];
    int ok = 1;
    if (pos0 < 0 || (long long)pos0 + S > (long long)max_pages * P) {
      atomicOr(status, kStatusAppendOverflow);
      ok = 0;
    }
    if (ok && cos_tab != nullptr && (long long)pos0 + S > rope_max_pos) {
      atomicOr(status, kStatusRopeRange);
      ok = 0;
    }
    s_pos0 = pos0;
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int pos0 = s_pos0;
  const bool rope = cos_tab != nullptr;
  const int half = d / 2;
  const int cpr = half / VEC;                 // chunks per half-row
  const int q_heads = (q_out != nullptr) ? Hq : 0;
  const int heads = q_heads + 2 * Hkv;        // q heads, then k heads, then v heads
  // q/k units pair the two halves (cpr units per head); v units copy (2*cpr per head).
  const int units_per_tok = (q_heads + Hkv) * cpr + Hkv * 2 * cpr;
  const long long total = (long long)S * units_per_tok;
  const int32_t* bt = block_table + (long long)b * max_pages;
  (void)heads;

  for (long long u = threadIdx.x; u < total; u += blockDim.x) {
    const int s = (int)(u / units_per_tok);
    int r = (int)(u - (long long)s * units_per_tok);
    const int pos = pos0 + s;
    const int page = bt[pos / P];
    const int slot = pos % P;
    if (page < 0 || page >= num_pages) {
      atomicOr(status, kStatusBadPage);
      continue;
    }
    if (r < (q_heads + Hkv) * cpr) {
      // RoPE pair unit for a q head (h < q_heads) or a k head.
      const int h = r / cpr;
      const int i = (r - h * cpr) * VEC;       // element offset in the first half
      const bool is_q = h < q_heads;
      const T* src = is_q ? q_in + (((long long)b * Hq + h) * S + s) * d
                          : k_in + (((long long)b * Hkv + (h - q_heads)) * S + s) * d;
      T* dst = is_q ? q_out + (((long long)b * Hq + h) * S + s) * d
                    : k_pages + (((long long)page * Hkv + (h - q_heads)) * P + slot) * d;
      Vec x1v = *reinterpret_cast<const Vec*>(src + i);
      Vec x2v = *reinterpret_cast<const Vec*>(src + i + half);
      if (rope) {
        // emb = cat(freqs, freqs) (rotary.py:67-68): both halves use columns i..i+VEC.
        const Vec cv = *reinterpret_cast<const Vec*>(cos_tab + (long long)pos * d + i);
        const Vec sv = *reinterpret_cast<const Vec*>(sin_tab + (long long)pos * d + i);
        const T* x1 = reinterpret_cast<const T*>(&x1v);
        const T* x2 = reinterpret_cast<const T*>(&x2v);
        const T* c = reinterpret_cast<const T*>(&cv);
        const T* sn = reinterpret_cast<const T*>(&sv);
        Vec o1v, o2v;
        T* o1 = reinterpret_cast<T*>(&o1v);
        T* o2 = reinterpret_cast<T*>(&o2v);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          o1[e] = rope_elem<T>(x1[e], x2[e], c[e], sn[e], true);
          o2[e] = rope_elem<T>(x2[e], x1[e], c[e], sn[e], false);
        }
        x1v = o1v;
        x2v = o2v;
      }
      *reinterpret_cast<Vec*>(dst + i) = x1v;
      *reinterpret_cast<Vec*>(dst + i + half) = x2v;
    } else {
      r -= (q_heads + Hkv) * cpr;
      const int h = r / (2 * cpr);
      const int i = (r - h * 2 * cpr) * VEC;
      const T* src = v_in + (((long long)b * Hkv + h) * S + s) * d;
      T* dst = v_pages + (((long long)page * Hkv + h) * P + slot) * d;
      *reinterpret_cast<Vec*>(dst + i) = *reinterpret_cast<const Vec*>(src + i);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) seq_lens[b] = pos0 + S;
}

template <typename T>
static cudaError_t launch_rope_append_t(const void* q_in, const void* k_in, const void* v_in,
                                        void* q_out, void* k_pages, void* v_pages,
                                        const int32_t* bt, int32_t* seq_lens, const void* cos_tab,
                                        const void* sin_tab, int B, int S, int Hq, int Hkv, int d,
                                        int P, int max_pages, int num_pages, int rope_max_pos,
                                        int32_t* status, cudaStream_t stream) {
  constexpr int V16 = 16 / sizeof(T);
  const int half = d / 2;
  auto aligned = [](const void* p, int a) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) % a) == 0; };
  const bool vec_ok = (half % V16) == 0 && aligned(q_in, 16) && aligned(k_in, 16) &&
                      aligned(v_in, 16) && aligned(q_out, 16) && aligned(k_pages, 16) &&
                      aligned(v_pages, 16) && aligned(cos_tab, 16) && aligned(sin_tab, 16);
  dim3 grid(B), block(512);
  if (vec_ok) {
    rope_append_kernel<T, V16><<<grid, block, 0, stream>>>(
        (const T*)q_in, (const T*)k_in, (const T*)v_in, (T*)q_out, (T*)k_pages, (T*)v_pages, bt,
        seq_lens, (const T*)cos_tab, (const T*)sin_tab, S, Hq, Hkv, d, P, max_pages, num_pages,
        rope_max_pos, status);
  } else {
    rope_append_kernel<T, 1><<<grid, block, 0, stream>>>(
        (const T*)q_in, (const T*)k_in, (const T*)v_in, (T*)q_out, (T*)k_pages, (T*)v_pages, bt,
        seq_lens, (const T*)cos_tab, (const T*)sin_tab, S, Hq, Hkv, d, P, max_pages, num_pages,
        rope_max_pos, status);
  }
  return cudaGetLastError();
}

cudaError_t launch_rope_append(const void* q_in, const void* k_in, const void* v_in, void* q_out,
                               void* k_pages, void* v_pages, const int32_t* bt, int32_t* seq_lens,
                               const void* cos_tab, const void* sin_tab, int B, int S, int Hq,
                               int Hkv, int d, int P, int max_pages, int num_pages,
                               int rope_max_pos, int dtype, int32_t* status,
                               cudaStream_t stream) {
  switch (dtype) {
    case LLMC_F32:
      return launch_rope_append_t<float>(q_in, k_in, v_in, q_out, k_pages, v_pages, bt, seq_lens,
                                         cos_tab, sin_tab, B, S, Hq, Hkv, d, P, max_pages,
                                         num_pages, rope_max_pos, status, stream);
    case LLMC_F16:
      return launch_rope_append_t<__half>(q_in, k_in, v_in, q_out, k_pages, v_pages, bt, seq_lens,
                                          cos_tab, sin_tab, B, S, Hq, Hkv, d, P, max_pages,
                                          num_pages, rope_max_pos, status, stream);
    default:
      return launch_rope_append_t<__nv_bfloat16>(q_in, k_in, v_in, q_out, k_pages, v_pages, bt,
                                                 seq_lens, cos_tab, sin_tab, B, S, Hq, Hkv, d, P,
                                                 max_pages, num_pages, rope_max_pos, status,
                                                 stream);
  }
}

}  // namespace llmc
