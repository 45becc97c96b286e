// Shared device helpers for the sm_100a decode-attention kernels.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a): mbarrier
// pipelines, TMA (cp.async.bulk.tensor) tile loads, ldmatrix/movmatrix and the
// m16n8k16 tensor-core MMA.  No CUTLASS/CuTe, no library kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/llm_cuda_b200.h"

namespace llmc {

// Counter words at the head of the balanced split's part_lse buffer: one per row
// (sequence, KV head, head group) plus a CTA counter, padded to 128 bytes.
__host__ __device__ __forceinline__ int balanced_counter_words(int rows) {
  return ((rows + 1) + 31) & ~31;
}


// Status bits written (atomicOr) into the caller's device status word.  The
// host reads the word after synchronising and raises; kernels never trap.
enum StatusBits : int {
  kStatusWaitTimeout = 1,      // a pipeline wait ran past its deadline
  kStatusBadPage = 2,          // block-table entry outside [0, num_pages)
  kStatusAppendOverflow = 4,   // append past max_pages_per_seq * page_size
  kStatusRopeRange = 8,        // RoPE position outside the cos/sin table
  kStatusSeqLenRange = 16,     // seq_len larger than the block table can address
};

// Every bounded wait gives up after this many nanoseconds of %globaltimer.
constexpr unsigned long long kWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false
// (and raises the CTA abort flag plus the device status bit) on timeout, or
// immediately once another warp of the CTA has aborted.  Never traps or spins
// without limit.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile int* abort_flag, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1;
      atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}

// Make generic-proxy writes to shared memory ordered before later async-proxy
// (TMA) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA: 2-D tiled bulk tensor load global -> shared, completing on an mbarrier.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start before its predecessor finishes;
// pdl_wait() blocks until the predecessor grid has completed and its memory is
// visible.  pdl_launch_dependents() lets the next such kernel start its prologue.
// Both are no-ops for kernels launched without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// cp.async (4-byte, global -> shared) for small index prefetches
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// ldmatrix / movmatrix / mma.sync m16n8k16
// ---------------------------------------------------------------------------
// ldmatrix reads shared memory that TMA filled: keep these volatile with a memory
// clobber so they never move above the mbarrier wait.  mma is a pure register op.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <typename T>
struct Mma;

template <>
struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

template <>
struct Mma<__half> {
  __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0,
                                             uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
};

// ---------------------------------------------------------------------------
// Element conversion
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Attention score with the reference's torch rounding (attention.py:67 of llm-cuda):
// torch.matmul(q, k^T) is rounded to the tensor dtype, then "/ sqrt(d)" is computed
// in fp32 and rounded again.  For fp32 both roundings are the identity.  The division
// is a multiplication by the fp32 reciprocal here; the two differ only when the fp32
// quotient lies within one fp32 ulp of a 16-bit rounding boundary.
template <typename T>
__device__ __forceinline__ float ref_score(float qk, float scale) {
  const float a = to_f32(from_f32<T>(qk));
  return to_f32(from_f32<T>(__fmul_rn(a, scale)));
}

// One RoPE output element with the reference's torch rounding (rotary.py:104-109):
// first half  x*cos + (-x_partner)*sin, second half x*cos + x_partner*sin; each
// product and the sum are rounded to T (no FMA contraction).
template <typename T>
__device__ __forceinline__ T rope_elem(T x_self, T x_partner, T c, T s, bool first_half) {
  const float xs = to_f32(x_self);
  const float xp = first_half ? -to_f32(x_partner) : to_f32(x_partner);
  const T a = from_f32<T>(__fmul_rn(xs, to_f32(c)));
  const T b = from_f32<T>(__fmul_rn(xp, to_f32(s)));
  return from_f32<T>(__fadd_rn(to_f32(a), to_f32(b)));
}

// Rotate two packed pairs (x1 = elements i, i+1 of the first half; x2 = the same
// elements of the second half) with packed cos/sin pairs of columns i, i+1.
template <typename T>
__device__ __forceinline__ void rope_pair2(uint32_t& x1, uint32_t& x2, uint32_t cs, uint32_t sn) {
  T* a = reinterpret_cast<T*>(&x1);
  T* b = reinterpret_cast<T*>(&x2);
  const T* c = reinterpret_cast<const T*>(&cs);
  const T* s = reinterpret_cast<const T*>(&sn);
  T o1[2], o2[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    o1[e] = rope_elem<T>(a[e], b[e], c[e], s[e], true);
    o2[e] = rope_elem<T>(b[e], a[e], c[e], s[e], false);
  }
  x1 = *reinterpret_cast<uint32_t*>(o1);
  x2 = *reinterpret_cast<uint32_t*>(o2);
}

}  // namespace llmc
