// C ABI of the decode-attention hot path (declared in include/llm_cuda_b200.h).
//
// Host-side argument validation happens here, before any launch; errors are
// reported as negative return codes plus a per-thread message, never by
// throwing across the ABI.
#include <climits>
#include <cstring>
#include <string>

#include "common.cuh"

namespace llmc {
cudaError_t launch_rope_append(const void* q_in, const void* k_in, const void* v_in, void* q_out,
                               void* k_pages, void* v_pages, const int32_t* bt, int32_t* seq_lens,
                               const void* cos_tab, const void* sin_tab, int B, int S, int Hq,
                               int Hkv, int d, int P, int max_pages, int num_pages,
                               int rope_max_pos, int dtype, int32_t* status, cudaStream_t stream);
cudaError_t launch_paged_decode(const void* q, const void* kp, const void* vp, const int32_t* bt,
                                const int32_t* seq_lens, void* out, float* part_o,
                                float* part_lse, int32_t* status, int B, int Hq, int Hkv, int D,
                                int P, int max_pages, int num_pages, int Tpart, float scale,
                                int dtype, int flags, std::string* err, cudaStream_t stream);
cudaError_t launch_lse_merge(const float* part_o, const float* part_lse, const int32_t* seq_lens,
                             void* out, int B, int Hq, int D, int max_parts, int Tpart, int cap,
                             int dtype, cudaStream_t stream);
cudaError_t launch_fused_decode(const void* q_raw, const void* k_new, const void* v_new,
                                void* q_rot_out, void* kp, void* vp, const int32_t* bt,
                                int32_t* seq_lens, const void* cos_tab, const void* sin_tab,
                                int rope_max_pos, void* out, float* part_o, float* part_lse,
                                int32_t* lens_next, int32_t* status, int B, int Hq, int Hkv,
                                int D, int P, int max_pages, int num_pages, int Tpart,
                                float scale, int dtype, std::string* err, cudaStream_t stream,
                                long long q_stride, long long kv_stride, int flags);
cudaError_t launch_decode_gemm(const void* x, const void* w, void* y, float* ws, size_t ws_floats,
                               int32_t* counters, int Mb, int N, int K, int32_t* status,
                               std::string* err, cudaStream_t stream);
size_t decode_gemm_workspace_floats(int Mb, int N, int K);
int balanced_grid();
bool fast_path_applies(int dtype, int D, int P, int max_pages, int Tpart, int B,
                       const void* q, const void* kp, const void* vp);
cudaError_t launch_add_rmsnorm(void* x, const void* delta, const void* w, void* h, int rows,
                               int hidden, float eps, int dtype, cudaStream_t stream);
cudaError_t launch_swiglu(const void* gu, void* out, int rows, int inter, int dtype,
                          cudaStream_t stream);
cudaError_t launch_argmax(const void* x, int64_t* out, int rows, int n, int dtype,
                          unsigned long long* keys, int* counters, int sms, cudaStream_t stream);
namespace ar {
struct Params {
  const void* partial;
  void* const* recv;
  int32_t* const* flags;
  int32_t* epoch;
  void* x;
  const void* w;
  void* h;
  int32_t* status;
  int rank, world, rows, rows_cap, hidden;
  float eps;
};
}  // namespace ar
size_t ar_recv_bytes(int world, int rows_cap, int hidden, int elem);
size_t ar_flag_bytes(int world, int rows_cap);
cudaError_t launch_allreduce_add_rmsnorm(const ar::Params& p, int dtype, std::string* err,
                                         cudaStream_t stream);
}  // namespace llmc

namespace {
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where, const std::string& extra = "") {
  std::string msg = std::string(where) + ": " + cudaGetErrorString(e);
  if (!extra.empty()) msg += " (" + extra + ")";
  return fail(LLMC_ECUDA, msg);
}

bool valid_dtype(int dt) { return dt == LLMC_F32 || dt == LLMC_F16 || dt == LLMC_BF16; }
}  // namespace

namespace llmc {
// Lets other translation units of the library report through llmc_last_error_string.
void set_last_error(const std::string& msg) { g_last_error = msg; }
}  // namespace llmc

extern "C" {

const char* llmc_last_error_string(void) { return g_last_error.c_str(); }

const char* llmc_version(void) { return "llm_cuda_b200 0.1.0 (sm_100a)"; }

int llmc_num_partitions(int max_tokens, int partition_tokens) {
  if (max_tokens <= 0 || partition_tokens <= 0) return 0;
  return (max_tokens + partition_tokens - 1) / partition_tokens;
}

size_t llmc_decode_partials_bytes(int B, int Hq, int d, int max_parts, size_t* lse_bytes) {
  const size_t rows = (size_t)(B > 0 ? B : 0) * (Hq > 0 ? Hq : 0) * (max_parts > 0 ? max_parts : 0);
  if (lse_bytes) *lse_bytes = rows * sizeof(float);
  return rows * (size_t)(d > 0 ? d : 0) * sizeof(float);
}

size_t llmc_balanced_partials_bytes(int B, int Hq, int Hkv, int d, size_t* lse_bytes) {
  if (B < 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || d <= 0) {
    if (lse_bytes) *lse_bytes = 0;
    return 0;
  }
  const size_t rows = (size_t)B * Hkv * ((Hq / Hkv + 7) / 8);
  const size_t slots = rows + (size_t)llmc::balanced_grid();
  const size_t counters = (size_t)llmc::balanced_counter_words((int)rows);
  if (lse_bytes) *lse_bytes = (counters + slots * 8) * sizeof(float);
  return slots * 8 * (size_t)d * sizeof(float);
}

int llmc_decode_balanced_supported(const void* q, const void* k_pages, const void* v_pages,
                                   int dtype, int d, int page_size, int max_pages_per_seq,
                                   int B) {
  return llmc::fast_path_applies(dtype, d, page_size, max_pages_per_seq, 0, B, q, k_pages,
                                 v_pages) ? 1 : 0;
}

int llmc_rope_append(const void* q_in, const void* k_in, const void* v_in, void* q_out,
                     void* k_pages, void* v_pages, const int32_t* block_table, int32_t* seq_lens,
                     const void* cos_tab, const void* sin_tab, int B, int S, int Hq, int Hkv,
                     int d, int page_size, int max_pages_per_seq, int num_pages, int rope_max_pos,
                     int dtype, int32_t* status, llmc_stream_t stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_rope_append: unknown dtype");
  if (B < 0 || S < 0 || Hkv <= 0 || Hq < 0 || d <= 0 || page_size <= 0 || max_pages_per_seq <= 0 ||
      num_pages <= 0)
    return fail(LLMC_EINVAL, "llmc_rope_append: sizes must be positive");
  if (d % 2) return fail(LLMC_EINVAL, "llmc_rope_append: head_dim must be even (rotate_half)");
  if ((cos_tab == nullptr) != (sin_tab == nullptr))
    return fail(LLMC_EINVAL, "llmc_rope_append: cos_tab and sin_tab must both be set or both NULL");
  if (cos_tab && rope_max_pos <= 0)
    return fail(LLMC_EINVAL, "llmc_rope_append: rope_max_pos must be positive with a table");
  if ((q_out == nullptr) != (q_in == nullptr))
    return fail(LLMC_EINVAL, "llmc_rope_append: q_in and q_out must both be set or both NULL");
  if (!k_in || !v_in || !k_pages || !v_pages || !block_table || !seq_lens || !status)
    return fail(LLMC_EINVAL, "llmc_rope_append: NULL pointer argument");
  if (B == 0 || S == 0) return LLMC_OK;
  cudaError_t e = llmc::launch_rope_append(q_in, k_in, v_in, q_out, k_pages, v_pages, block_table,
                                           seq_lens, cos_tab, sin_tab, B, S, Hq, Hkv, d,
                                           page_size, max_pages_per_seq, num_pages, rope_max_pos,
                                           dtype, status, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_rope_append");
  return LLMC_OK;
}

int llmc_paged_decode(const void* q, const void* k_pages, const void* v_pages,
                      const int32_t* block_table, const int32_t* seq_lens, void* out,
                      float* part_o, float* part_lse, int32_t* status, int B, int Hq, int Hkv,
                      int d, int page_size, int max_pages_per_seq, int num_pages,
                      int partition_tokens, float scale, int dtype, int flags,
                      llmc_stream_t stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_paged_decode: unknown dtype");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || d <= 0 || page_size <= 0 || max_pages_per_seq <= 0 ||
      num_pages <= 0 || partition_tokens < 0)
    return fail(LLMC_EINVAL, "llmc_paged_decode: sizes must be positive");
  if (Hq % Hkv) return fail(LLMC_EINVAL, "llmc_paged_decode: Hq must be a multiple of Hkv");
  if (d > 256) return fail(LLMC_EUNSUPPORTED, "llmc_paged_decode: head_dim > 256");
  if (partition_tokens % 64)
    return fail(LLMC_EINVAL, "llmc_paged_decode: partition_tokens must be a multiple of 64");
  if ((long long)Hq / Hkv * d > 16384)
    return fail(LLMC_EUNSUPPORTED, "llmc_paged_decode: (Hq/Hkv) * head_dim > 16384");
  if ((long long)num_pages * Hkv * page_size >= (1ll << 31))
    return fail(LLMC_EUNSUPPORTED, "llmc_paged_decode: page pool rows exceed 2^31");
  if (!q || !k_pages || !v_pages || !block_table || !seq_lens || !out || !status)
    return fail(LLMC_EINVAL, "llmc_paged_decode: NULL pointer argument");
  const long long cap_tokens = (long long)max_pages_per_seq * page_size;
  if (cap_tokens > INT_MAX)
    return fail(LLMC_EINVAL, "llmc_paged_decode: max_pages_per_seq * page_size exceeds 2^31-1");
  const int max_parts = llmc_num_partitions((int)cap_tokens, partition_tokens);
  if ((partition_tokens == 0 || max_parts > 1) && (!part_o || !part_lse))
    return fail(LLMC_EINVAL,
                "llmc_paged_decode: part_o/part_lse are required when a sequence can span "
                "more than one partition");
  std::string err;
  cudaError_t e = llmc::launch_paged_decode(q, k_pages, v_pages, block_table, seq_lens, out,
                                            part_o, part_lse, status, B, Hq, Hkv, d, page_size,
                                            max_pages_per_seq, num_pages, partition_tokens, scale,
                                            dtype, flags, &err, (cudaStream_t)stream);
  if (e == cudaErrorNotSupported && partition_tokens == 0)
    return fail(LLMC_EUNSUPPORTED, "llmc_paged_decode: " + err);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_paged_decode", err);
  return LLMC_OK;
}

int llmc_lse_merge(const float* part_o, const float* part_lse, const int32_t* seq_lens, void* out,
                   int B, int Hq, int d, int max_parts, int partition_tokens, int dtype,
                   llmc_stream_t stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_lse_merge: unknown dtype");
  if (B < 0 || Hq <= 0 || d <= 0 || partition_tokens < 0 ||
      (partition_tokens > 0 && max_parts <= 0))
    return fail(LLMC_EINVAL, "llmc_lse_merge: sizes must be positive");
  if (!seq_lens || !out) return fail(LLMC_EINVAL, "llmc_lse_merge: NULL pointer argument");
  if ((partition_tokens == 0 || max_parts > 1) && (!part_o || !part_lse))
    return fail(LLMC_EINVAL, "llmc_lse_merge: NULL partials with max_parts > 1");
  cudaError_t e = llmc::launch_lse_merge(part_o, part_lse, seq_lens, out, B, Hq, d, max_parts,
                                         partition_tokens, max_parts * partition_tokens, dtype,
                                         (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_lse_merge");
  return LLMC_OK;
}

int llmc_rope_append_decode_strided(
    const void* q, const void* k_new, const void* v_new, void* q_rot_out, void* k_pages,
    void* v_pages, const int32_t* block_table, int32_t* seq_lens, const void* cos_tab,
    const void* sin_tab, int rope_max_pos, void* out, float* part_o, float* part_lse,
    int32_t* lens_next, int32_t* status, int B, int Hq, int Hkv, int d, int page_size,
    int max_pages_per_seq, int num_pages, int partition_tokens, float scale, int dtype,
    long long q_seq_stride, long long kv_seq_stride, int flags, llmc_stream_t stream) {
  g_last_error.clear();
  const bool dense = q_seq_stride == (long long)Hq * d && kv_seq_stride == (long long)Hkv * d;
  if (q_seq_stride < (long long)Hq * d || kv_seq_stride < (long long)Hkv * d)
    return fail(LLMC_EINVAL, "llmc_rope_append_decode: sequence strides smaller than Hq*d / Hkv*d");
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_rope_append_decode: unknown dtype");
  if (B < 0 || Hq <= 0 || Hkv <= 0 || d <= 0 || page_size <= 0 || max_pages_per_seq <= 0 ||
      num_pages <= 0 || partition_tokens < 0 || rope_max_pos <= 0)
    return fail(LLMC_EINVAL, "llmc_rope_append_decode: sizes must be positive");
  if (Hq % Hkv) return fail(LLMC_EINVAL, "llmc_rope_append_decode: Hq must be a multiple of Hkv");
  if (d % 2 || d > 256)
    return fail(LLMC_EUNSUPPORTED, "llmc_rope_append_decode: head_dim must be even and <= 256");
  if (partition_tokens % 64)
    return fail(LLMC_EINVAL, "llmc_rope_append_decode: partition_tokens must be a multiple of 64");
  if ((long long)Hq / Hkv * d > 16384)
    return fail(LLMC_EUNSUPPORTED, "llmc_rope_append_decode: (Hq/Hkv) * head_dim > 16384");
  if ((long long)num_pages * Hkv * page_size >= (1ll << 31))
    return fail(LLMC_EUNSUPPORTED, "llmc_rope_append_decode: page pool rows exceed 2^31");
  if (!q || !k_new || !v_new || !q_rot_out || !k_pages || !v_pages || !block_table || !seq_lens ||
      !cos_tab || !sin_tab || !out || !lens_next || !status)
    return fail(LLMC_EINVAL, "llmc_rope_append_decode: NULL pointer argument");
  const long long cap_tokens = (long long)max_pages_per_seq * page_size;
  if (cap_tokens > INT_MAX)
    return fail(LLMC_EINVAL,
                "llmc_rope_append_decode: max_pages_per_seq * page_size exceeds 2^31-1");
  int max_parts = llmc_num_partitions((int)cap_tokens, partition_tokens);
  if ((partition_tokens == 0 || max_parts > 1) && (!part_o || !part_lse))
    return fail(LLMC_EINVAL, "llmc_rope_append_decode: part_o/part_lse are required");
  if (B == 0) return LLMC_OK;
  std::string err;
  cudaError_t e = llmc::launch_fused_decode(
      q, k_new, v_new, q_rot_out, k_pages, v_pages, block_table, seq_lens, cos_tab, sin_tab,
      rope_max_pos, out, part_o, part_lse, lens_next, status, B, Hq, Hkv, d, page_size,
      max_pages_per_seq, num_pages, partition_tokens, scale, dtype, &err, (cudaStream_t)stream,
      q_seq_stride, kv_seq_stride, flags);
  if (e == cudaErrorNotSupported && !dense)
    return fail(LLMC_EUNSUPPORTED,
                "llmc_rope_append_decode: strided q/k/v need the fused kernel's shapes");
  if (e == cudaErrorNotSupported) {
    // Shape outside the fused kernel: the same step with the separate kernels.
    cudaGetLastError();
    if (partition_tokens == 0) {
      // The balanced split needs the fused kernel; the SIMT kernel gets uniform
      // partitions, as many as the balanced workspace holds.
      // The uniform log-sum-exps go after the balanced split's counter words, so the
      // counters stay zero for a later balanced call on the same buffers.
      size_t lse_b = 0;
      const size_t o_b = llmc_balanced_partials_bytes(B, Hq, Hkv, d, &lse_b);
      const size_t cw = (size_t)llmc::balanced_counter_words(B * Hkv * ((Hq / Hkv + 7) / 8));
      const size_t lse_words = lse_b / sizeof(float) > cw ? lse_b / sizeof(float) - cw : 0;
      size_t per_part = 0;
      const size_t o1 = llmc_decode_partials_bytes(B, Hq, d, 1, &per_part);
      size_t fit = o1 ? o_b / o1 : 1;
      if (per_part && lse_words * sizeof(float) / per_part < fit)
        fit = lse_words * sizeof(float) / per_part;
      if (fit < 1) fit = 1;
      long long T = (cap_tokens + (long long)fit - 1) / (long long)fit;
      T = (T + 63) / 64 * 64;
      partition_tokens = (int)(T < (1ll << 30) ? T : (1ll << 30));
      max_parts = llmc_num_partitions((int)cap_tokens, partition_tokens);
      part_lse += cw;
    }
    int rc = llmc_rope_append(q, k_new, v_new, q_rot_out, k_pages, v_pages, block_table, seq_lens,
                              cos_tab, sin_tab, B, 1, Hq, Hkv, d, page_size, max_pages_per_seq,
                              num_pages, rope_max_pos, dtype, status, stream);
    if (rc) return rc;
    rc = llmc_paged_decode(q_rot_out, k_pages, v_pages, block_table, seq_lens, out, part_o,
                           part_lse, status, B, Hq, Hkv, d, page_size, max_pages_per_seq,
                           num_pages, partition_tokens, scale, dtype, 0, stream);
    if (rc) return rc;
    return llmc_lse_merge(part_o, part_lse, seq_lens, out, B, Hq, d, max_parts,
                          partition_tokens, dtype, stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "llmc_rope_append_decode", err);
  return LLMC_OK;
}

int llmc_rope_append_decode(const void* q, const void* k_new, const void* v_new, void* q_rot_out,
                            void* k_pages, void* v_pages, const int32_t* block_table,
                            int32_t* seq_lens, const void* cos_tab, const void* sin_tab,
                            int rope_max_pos, void* out, float* part_o, float* part_lse,
                            int32_t* lens_next, int32_t* status, int B, int Hq, int Hkv, int d,
                            int page_size, int max_pages_per_seq, int num_pages,
                            int partition_tokens, float scale, int dtype, llmc_stream_t stream) {
  return llmc_rope_append_decode_strided(
      q, k_new, v_new, q_rot_out, k_pages, v_pages, block_table, seq_lens, cos_tab, sin_tab,
      rope_max_pos, out, part_o, part_lse, lens_next, status, B, Hq, Hkv, d, page_size,
      max_pages_per_seq, num_pages, partition_tokens, scale, dtype, (long long)Hq * d,
      (long long)Hkv * d, 0, stream);
}

size_t llmc_decode_gemm_workspace_bytes(int Mb, int N, int K) {
  if (Mb <= 0 || Mb > 256 || N <= 0 || K <= 0 || N % 128 || K % 64) return 0;
  return llmc::decode_gemm_workspace_floats(Mb, N, K) * sizeof(float);
}

int llmc_decode_gemm(const void* x, const void* w, void* y, float* workspace,
                     size_t workspace_bytes, int32_t* counters, int Mb, int N, int K,
                     int32_t* status, llmc_stream_t stream) {
  g_last_error.clear();
  if (Mb <= 0 || Mb > 256 || N <= 0 || K <= 0)
    return fail(LLMC_EINVAL, "llmc_decode_gemm: need 1 <= Mb <= 256 and positive N, K");
  if (N % 128 || K % 64)
    return fail(LLMC_EUNSUPPORTED, "llmc_decode_gemm: N must be a multiple of 128, K of 64");
  if (!x || !w || !y || !workspace || !counters || !status)
    return fail(LLMC_EINVAL, "llmc_decode_gemm: NULL pointer");
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(x) || !al(w)) return fail(LLMC_EINVAL, "llmc_decode_gemm: x and W must be 16-byte aligned");
  std::string err;
  cudaError_t e = llmc::launch_decode_gemm(x, w, y, workspace, workspace_bytes / sizeof(float),
                                           counters, Mb, N, K, status, &err, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_decode_gemm", err);
  return LLMC_OK;
}

int llmc_add_rmsnorm(void* x, const void* delta, const void* weight, void* out, int rows,
                     int hidden, float eps, int dtype, llmc_stream_t stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_add_rmsnorm: unknown dtype");
  if (rows < 0 || hidden <= 0) return fail(LLMC_EINVAL, "llmc_add_rmsnorm: bad sizes");
  if (!x || !weight || !out) return fail(LLMC_EINVAL, "llmc_add_rmsnorm: NULL pointer argument");
  if (rows == 0) return LLMC_OK;
  cudaError_t e = llmc::launch_add_rmsnorm(x, delta, weight, out, rows, hidden, eps, dtype,
                                           (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_add_rmsnorm");
  return LLMC_OK;
}

int llmc_swiglu(const void* gate_up, void* out, int rows, int inter, int dtype,
                llmc_stream_t stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_swiglu: unknown dtype");
  if (rows < 0 || inter <= 0) return fail(LLMC_EINVAL, "llmc_swiglu: bad sizes");
  if (!gate_up || !out) return fail(LLMC_EINVAL, "llmc_swiglu: NULL pointer argument");
  if (rows == 0) return LLMC_OK;
  cudaError_t e = llmc::launch_swiglu(gate_up, out, rows, inter, dtype, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_swiglu");
  return LLMC_OK;
}

size_t llmc_argmax_workspace_bytes(int rows) {
  return rows > 0 ? (size_t)rows * (sizeof(unsigned long long) + sizeof(int)) : 0;
}

int llmc_argmax(const void* x, int64_t* out, int rows, int n, int dtype, void* workspace,
                llmc_stream_t stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_argmax: unknown dtype");
  if (rows < 0 || n <= 0 || rows > 65535) return fail(LLMC_EINVAL, "llmc_argmax: bad sizes");
  if (!x || !out || !workspace) return fail(LLMC_EINVAL, "llmc_argmax: NULL pointer argument");
  if (reinterpret_cast<uintptr_t>(workspace) & 7)
    return fail(LLMC_EINVAL, "llmc_argmax: workspace must be 8-byte aligned");
  if (rows == 0) return LLMC_OK;
  auto* keys = static_cast<unsigned long long*>(workspace);
  int* counters = reinterpret_cast<int*>(keys + rows);
  cudaError_t e = llmc::launch_argmax(x, out, rows, n, dtype, keys, counters,
                                      llmc::balanced_grid(), (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_argmax");
  return LLMC_OK;
}

size_t llmc_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int llmc_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  g_last_error.clear();
  if (!dev_ptr || !handle || bytes == 0) return fail(LLMC_EINVAL, "llmc_ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_ipc_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "llmc_ipc_alloc");
  }
  *dev_ptr = p;
  return LLMC_OK;
}

int llmc_ipc_open(const void* handle, void** dev_ptr) {
  g_last_error.clear();
  if (!handle || !dev_ptr) return fail(LLMC_EINVAL, "llmc_ipc_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_ipc_open");
  return LLMC_OK;
}

int llmc_ipc_close(void* dev_ptr) {
  g_last_error.clear();
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_ipc_close");
  return LLMC_OK;
}

int llmc_ipc_free(void* dev_ptr) {
  g_last_error.clear();
  cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_ipc_free");
  return LLMC_OK;
}

size_t llmc_ar_region_bytes(int world, int rows_cap, int hidden, int dtype, size_t* flag_bytes) {
  if (world <= 0 || rows_cap <= 0 || hidden <= 0 || !valid_dtype(dtype)) {
    if (flag_bytes) *flag_bytes = 0;
    return 0;
  }
  if (flag_bytes) *flag_bytes = llmc::ar_flag_bytes(world, rows_cap);
  return llmc::ar_recv_bytes(world, rows_cap, hidden, dtype == LLMC_F32 ? 4 : 2);
}

int llmc_allreduce_add_rmsnorm(const void* partial, void* const* recv_ptrs,
                               int32_t* const* flag_ptrs, int32_t* epoch, void* x,
                               const void* weight, void* out, int32_t* status, int rank,
                               int world, int rows, int rows_cap, int hidden, float eps,
                               int dtype, llmc_stream_t stream) {
  g_last_error.clear();
  if (!valid_dtype(dtype)) return fail(LLMC_EINVAL, "llmc_allreduce_add_rmsnorm: unknown dtype");
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return fail(LLMC_EINVAL, "llmc_allreduce_add_rmsnorm: need 0 <= rank < world <= 8");
  if (rows < 0 || rows > rows_cap || hidden <= 0)
    return fail(LLMC_EINVAL, "llmc_allreduce_add_rmsnorm: need 0 <= rows <= rows_cap, hidden > 0");
  if (!partial || !recv_ptrs || !epoch || !x || !weight || !out || !status)
    return fail(LLMC_EINVAL, "llmc_allreduce_add_rmsnorm: NULL pointer argument");
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(partial) || !al(x) || !al(weight) || !al(out))
    return fail(LLMC_EINVAL, "llmc_allreduce_add_rmsnorm: tensors must be 16-byte aligned");
  if (rows == 0) return LLMC_OK;
  llmc::ar::Params p;
  p.partial = partial; p.recv = recv_ptrs; p.flags = flag_ptrs; p.epoch = epoch;
  p.x = x; p.w = weight; p.h = out; p.status = status;
  p.rank = rank; p.world = world; p.rows = rows; p.rows_cap = rows_cap; p.hidden = hidden;
  p.eps = eps;
  std::string err;
  cudaError_t e = llmc::launch_allreduce_add_rmsnorm(p, dtype, &err, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "llmc_allreduce_add_rmsnorm", err);
  return LLMC_OK;
}

}  // extern "C"
