// llmc_paged_decode_noalloc: paged decode attention for callers that cannot
// allocate device memory.
//
// llmc_paged_decode needs a caller-provided split-K workspace (part_o/part_lse).
// Some callers cannot hand one over: code running where cudaMalloc is forbidden or
// unavailable (a host framework that owns all device memory and exposes no
// allocator hook, a plugin that may only touch the buffers it is given, or a
// process that must not allocate after start-up).  This entry point keeps that
// workspace in a fixed array compiled into the library instead, and launches the
// same decode and merge kernels as llmc_paged_decode + llmc_lse_merge.
//
// Limits and behaviour:
//  * The array holds kScratchFloats floats (8 MiB); every GPU that loads the
//    library keeps it until the process exits.  A call whose partials need more
//    (B * Hq * max_parts * (d + 1) floats) is rejected with LLMC_EINVAL.
//  * The first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * All calls share the one array and it keeps the previous call's contents.
//    Nothing in it needs to start at zero: each call writes every partial it
//    later reads.  Calls whose work overlaps on the GPU (other streams, other
//    host threads) race on the array; issue them in order on one stream.
//  * No cudaMalloc, cudaFree or other allocating routine is called.
#include <climits>
#include <mutex>
#include <string>

#include "common.cuh"

namespace llmc {
cudaError_t launch_paged_decode(const void* q, const void* kp, const void* vp, const int32_t* bt,
                                const int32_t* seq_lens, void* out, float* part_o,
                                float* part_lse, int32_t* status, int B, int Hq, int Hkv, int D,
                                int P, int max_pages, int num_pages, int Tpart, float scale,
                                int dtype, int flags, std::string* err, cudaStream_t stream);
cudaError_t launch_lse_merge(const float* part_o, const float* part_lse, const int32_t* seq_lens,
                             void* out, int B, int Hq, int D, int max_parts, int Tpart, int cap,
                             int dtype, cudaStream_t stream);
void set_last_error(const std::string& msg);
}  // namespace llmc

namespace {
constexpr size_t kScratchFloats = size_t(2) << 20;  // 8 MiB of fp32 partials
static __device__ __align__(256) float g_decode_scratch[kScratchFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of g_decode_scratch on the current device (looked up once per device).
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

int fail(int code, const std::string& msg) {
  llmc::set_last_error(msg);
  return code;
}
}  // namespace

extern "C" {

LLMC_API size_t llmc_paged_decode_noalloc_capacity_bytes(void) {
  return kScratchFloats * sizeof(float);
}

LLMC_API int llmc_paged_decode_noalloc(const void* q, const void* k_pages, const void* v_pages,
                                       const int32_t* block_table, const int32_t* seq_lens,
                                       void* out, int32_t* status, int B, int Hq, int Hkv, int d,
                                       int page_size, int max_pages_per_seq, int num_pages,
                                       int partition_tokens, float scale, int dtype,
                                       llmc_stream_t stream) {
  llmc::set_last_error("");
  if (dtype != LLMC_F32 && dtype != LLMC_F16 && dtype != LLMC_BF16)
    return fail(LLMC_EINVAL, "llmc_paged_decode_noalloc: unknown dtype");
  if (partition_tokens == LLMC_PARTITION_BALANCED)
    return fail(LLMC_EINVAL,
                "llmc_paged_decode_noalloc: the balanced split (partition_tokens 0) is not "
                "supported here; pass a positive multiple of 64");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || d <= 0 || page_size <= 0 || max_pages_per_seq <= 0 ||
      num_pages <= 0 || partition_tokens < 0)
    return fail(LLMC_EINVAL, "llmc_paged_decode_noalloc: sizes must be positive");
  if (Hq % Hkv) return fail(LLMC_EINVAL, "llmc_paged_decode_noalloc: Hq must be a multiple of Hkv");
  if (d > 256) return fail(LLMC_EUNSUPPORTED, "llmc_paged_decode_noalloc: head_dim > 256");
  if (partition_tokens % 64)
    return fail(LLMC_EINVAL,
                "llmc_paged_decode_noalloc: partition_tokens must be a multiple of 64");
  if ((long long)Hq / Hkv * d > 16384)
    return fail(LLMC_EUNSUPPORTED, "llmc_paged_decode_noalloc: (Hq/Hkv) * head_dim > 16384");
  if ((long long)num_pages * Hkv * page_size >= (1ll << 31))
    return fail(LLMC_EUNSUPPORTED, "llmc_paged_decode_noalloc: page pool rows exceed 2^31");
  if (!q || !k_pages || !v_pages || !block_table || !seq_lens || !out || !status)
    return fail(LLMC_EINVAL, "llmc_paged_decode_noalloc: NULL pointer argument");
  const long long cap_tokens = (long long)max_pages_per_seq * page_size;
  if (cap_tokens > INT_MAX)
    return fail(LLMC_EINVAL,
                "llmc_paged_decode_noalloc: max_pages_per_seq * page_size exceeds 2^31-1");
  const int max_parts = (int)((cap_tokens + partition_tokens - 1) / partition_tokens);
  const size_t rows = (size_t)B * Hq * max_parts;
  const size_t need = rows * (size_t)d + rows;
  if (need > kScratchFloats)
    return fail(LLMC_EINVAL,
                "llmc_paged_decode_noalloc: split-K partials need " + std::to_string(need * 4) +
                    " bytes, more than the built-in " + std::to_string(kScratchFloats * 4) +
                    "-byte scratch; raise partition_tokens or use llmc_paged_decode");
  if (B == 0) return LLMC_OK;
  float* scratch = nullptr;
  cudaError_t e = scratch_for_current_device(&scratch);
  if (e != cudaSuccess)
    return fail(LLMC_ECUDA, std::string("llmc_paged_decode_noalloc: scratch lookup: ") +
                                cudaGetErrorString(e));
  float* part_o = scratch;
  float* part_lse = scratch + rows * (size_t)d;
  std::string err;
  e = llmc::launch_paged_decode(q, k_pages, v_pages, block_table, seq_lens, out, part_o, part_lse,
                                status, B, Hq, Hkv, d, page_size, max_pages_per_seq, num_pages,
                                partition_tokens, scale, dtype, 0, &err, (cudaStream_t)stream);
  if (e != cudaSuccess)
    return fail(LLMC_ECUDA, std::string("llmc_paged_decode_noalloc: decode: ") +
                                cudaGetErrorString(e) + (err.empty() ? "" : " (" + err + ")"));
  e = llmc::launch_lse_merge(part_o, part_lse, seq_lens, out, B, Hq, d, max_parts,
                             partition_tokens, max_parts * partition_tokens, dtype,
                             (cudaStream_t)stream);
  if (e != cudaSuccess)
    return fail(LLMC_ECUDA, std::string("llmc_paged_decode_noalloc: merge: ") +
                                cudaGetErrorString(e));
  return LLMC_OK;
}

}  // extern "C"
