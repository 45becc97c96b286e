/*
 * llm_cuda_b200 — C ABI of the B200 (sm_100a) decode-attention hot path.
 *
 * Every pointer argument is a DEVICE pointer owned by the caller; no entry point
 * allocates device memory.  Tensors are dense row-major in the layouts given
 * below.  Work is enqueued on `stream` and nothing synchronises the host, so the
 * calls can be captured in a CUDA graph.  Return value: LLMC_OK (0) on success, a
 * negative LLMC_E* code otherwise (argument validation happens on the host before
 * any launch; `llmc_last_error_string()` holds the message, per host thread).
 *
 * Device-side faults are never raised by trapping: kernels OR bits into the
 * caller's `status` word (int32 in device memory, see LLMC_STATUS_*), which the
 * caller reads after synchronising.
 *
 * Paths below are files of the calvin-fei/llm-cuda project.
 */
#ifndef LLM_CUDA_B200_H_
#define LLM_CUDA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* llmc_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define LLMC_API __attribute__((visibility("default")))
#else
#define LLMC_API
#endif

/* Element types (the tensor dtype of q/k/v/out, pages and cos/sin tables). */
#define LLMC_F32 0
#define LLMC_F16 1
#define LLMC_BF16 2

#define LLMC_OK 0
#define LLMC_EINVAL (-1)     /* invalid argument                            */
#define LLMC_EUNSUPPORTED (-2) /* shape/dtype combination not supported     */
#define LLMC_ECUDA (-3)      /* CUDA runtime/driver error at launch         */

/* Bits of the device status word. */
#define LLMC_STATUS_WAIT_TIMEOUT 1
#define LLMC_STATUS_BAD_PAGE 2
#define LLMC_STATUS_APPEND_OVERFLOW 4
#define LLMC_STATUS_ROPE_RANGE 8
#define LLMC_STATUS_SEQLEN_RANGE 16

/* llmc_paged_decode / llmc_rope_append_decode_strided flags */
#define LLMC_DECODE_FORCE_GENERIC 1 /* use the SIMT kernel even where the TMA kernel applies */
/*
 * LLMC_DECODE_EARLY_TABLES (balanced split only; ignored otherwise): the caller
 * guarantees that seq_lens, block_table and the page pools are not written by any
 * kernel that can still be running when this launch begins under programmatic
 * dependent launch (the kernel just before it on the stream, or one before that which
 * it has let start early).  The kernel then scans the lengths, splits the work and
 * starts streaming K/V before it waits for the previous kernel; only the query, the
 * new token's k/v and every write wait.  A decode step whose tables are touched only
 * by this layer's own launch (and by the host between steps) qualifies.
 */
#define LLMC_DECODE_EARLY_TABLES 2

/*
 * Fused RoPE-on-new-tokens + KV-page append.
 *
 * Replaces, per decode step, the reference's
 *   build_rope_cache + apply_rotary   (src/llm_cuda/models/llama3/attention.py:110-119,
 *                                      src/llm_cuda/models/llama3/rotary.py:29-109,
 *                                      src/llm_cuda/kernels/triton/rope.py:156-222)
 *   PagedKVLayerCache.append          (src/llm_cuda/models/llama3/kv_cache.py:38-63)
 * and generalises the cache to a block table over a shared page pool, batch B.
 *
 *   q_in   [B, Hq,  S, d]  raw query of the S new tokens (may be NULL with q_out NULL)
 *   k_in   [B, Hkv, S, d]  raw key   (rotated before it is stored)
 *   v_in   [B, Hkv, S, d]  value
 *   q_out  [B, Hq,  S, d]  rotated query (NULL: not produced)
 *   k_pages, v_pages [num_pages, Hkv, page_size, d]  the page pools (written)
 *   block_table [B, max_pages_per_seq] int32 physical page of each logical page
 *   seq_lens [B] int32: token s of sequence b lands at position seq_lens[b] + s;
 *            on return seq_lens[b] has grown by S (updated on the device)
 *   cos_tab, sin_tab [rope_max_pos, d] in the tensor dtype, rows indexed by position,
 *            as built by build_rope_cache (rotary.py:29-71).  Both NULL: no rotation
 *            (plain append of already-rotated k, as PagedKVLayerCache.append does).
 * Rounding follows the reference's torch path (rotary.py:104-109): x*cos and
 * rotate_half(x)*sin are each rounded to the dtype, then their sum.
 */
LLMC_API int llmc_rope_append(const void* q_in, const void* k_in, const void* v_in, void* q_out,
                     void* k_pages, void* v_pages, const int32_t* block_table, int32_t* seq_lens,
                     const void* cos_tab, const void* sin_tab, int B, int S, int Hq, int Hkv,
                     int d, int page_size, int max_pages_per_seq, int num_pages, int rope_max_pos,
                     int dtype, int32_t* status, llmc_stream_t stream);

/*
 * Workspace for split-K partials of llmc_paged_decode / llmc_lse_merge:
 * part_o float32 [B, Hq, max_parts, d] then part_lse float32 [B, Hq, max_parts].
 * Returns the number of BYTES of part_o (first) and, via *lse_bytes, of part_lse.
 */
LLMC_API size_t llmc_decode_partials_bytes(int B, int Hq, int d, int max_parts, size_t* lse_bytes);

/* Number of partitions a context of `max_tokens` is split into at `partition_tokens`. */
LLMC_API int llmc_num_partitions(int max_tokens, int partition_tokens);

/*
 * partition_tokens == LLMC_PARTITION_BALANCED selects the balanced split of the TMA
 * kernel.  It has no counterpart in the reference, which has no split-K.
 *  - The 64-token chunks of all (sequence, KV head) rows are laid end to end, and
 *    CTA c of the G = SM-count grid takes chunks [c*total/G, (c+1)*total/G).
 *  - Every SM gets the same number of tokens whatever the lengths. The split is
 *    computed on the device from seq_lens, so a captured graph stays balanced as
 *    contexts grow.
 *  - Rows that one CTA covers entirely go straight to out. The others leave one
 *    partial per CTA, and the CTA that completes a row's last partial merges the row.
 *    The decode launch thus finishes out by itself, and llmc_lse_merge with
 *    partition_tokens 0 does nothing.
 *  - The partials buffers are sized by llmc_balanced_partials_bytes on the device that
 *    runs the kernels.
 *  - part_lse begins with counter words, one per row plus one. These must be zero
 *    before a call: zero the buffer when it is allocated, when (B, Hq, Hkv) changes,
 *    and after a call that reported LLMC_STATUS_WAIT_TIMEOUT. Every completed call
 *    leaves them at zero.
 *  - llmc_paged_decode returns LLMC_EUNSUPPORTED where the TMA kernel does not apply
 *    (see llmc_decode_balanced_supported). llmc_rope_append_decode then falls back to
 *    uniform partitions that fit the same buffers; their log-sum-exps are stored after
 *    the counter words, which stay zero.
 */
#define LLMC_PARTITION_BALANCED 0

/* Bytes of part_o (returned) and part_lse (*lse_bytes) for the balanced split. */
LLMC_API size_t llmc_balanced_partials_bytes(int B, int Hq, int Hkv, int d, size_t* lse_bytes);

/* 1 if llmc_paged_decode takes LLMC_PARTITION_BALANCED for these arguments, else 0. */
LLMC_API int llmc_decode_balanced_supported(const void* q, const void* k_pages,
                                            const void* v_pages, int dtype, int d,
                                            int page_size, int max_pages_per_seq, int B);

/*
 * Paged GQA flash-decode: one query token per sequence against its paged K/V.
 *
 * Replaces triton_decode_attention / _decode_attention_kernel
 * (src/llm_cuda/kernels/triton/decode_attention.py:47-159, 204-287) and the
 * get_kv gather feeding it (src/llm_cuda/models/llama3/kv_cache.py:65-83): the
 * kernel reads pages in place through the block table.  Query head h uses KV
 * head h / (Hq / Hkv) (decode_attention.py:90-93); out = softmax(q.K^T * scale).V
 * with out = acc / max(l, 1e-9) (decode_attention.py:154).
 *
 *   q   [B, Hq, d]; out [B, Hq, d] (same dtype)
 *   k_pages, v_pages [num_pages, Hkv, page_size, d]
 *   block_table [B, max_pages_per_seq] int32; seq_lens [B] int32 (tokens to attend)
 *   partition_tokens: split-K bound T (multiple of 64), or LLMC_PARTITION_BALANCED.
 *     With T > 0 a context of L tokens is cut
 *     into n = ceil(L / T) partitions of equal length (L / n rounded up to 64).
 *     Sequences with n > 1 leave normalised partials + log2-sum-exp in part_o/part_lse
 *     for llmc_lse_merge; single-partition sequences are written to out directly.
 *   part_o/part_lse: see llmc_decode_partials_bytes with
 *     max_parts = llmc_num_partitions(max_pages_per_seq * page_size, partition_tokens);
 *     may be NULL when max_parts == 1.
 *   flags: LLMC_DECODE_FORCE_GENERIC, LLMC_DECODE_EARLY_TABLES (ORed), or 0.
 * The hot kernel (bf16/fp16, d in {64,128,256}) is a persistent TMA + mbarrier
 * pipeline with tensor-core (mma.sync) tiles, one CTA per SM; other shapes use a
 * SIMT kernel with the same partial format.
 */
LLMC_API int llmc_paged_decode(const void* q, const void* k_pages, const void* v_pages,
                      const int32_t* block_table, const int32_t* seq_lens, void* out,
                      float* part_o, float* part_lse, int32_t* status, int B, int Hq, int Hkv,
                      int d, int page_size, int max_pages_per_seq, int num_pages,
                      int partition_tokens, float scale, int dtype, int flags,
                      llmc_stream_t stream);

/*
 * One decode step of attention with RoPE and the KV-page append fused in:
 * llmc_rope_append (S = 1) + llmc_paged_decode + llmc_lse_merge in two launches.
 *
 * Replaces the decode branch of Llama3Attention.forward between the projections and
 * o_proj (src/llm_cuda/models/llama3/attention.py:110-139): build_rope_cache +
 * apply_rotary (rotary.py:29-109), PagedKVLayerCache.append (kv_cache.py:38-63),
 * get_kv (kv_cache.py:65-83) and triton_decode_attention (decode_attention.py:204-287).
 *
 *   q [B, Hq, d] raw (un-rotated) query of the new token; k_new, v_new [B, Hkv, d].
 *   seq_lens [B]: lengths BEFORE the step; the new token goes to position seq_lens[b]
 *     and on completion seq_lens[b] has grown by one (written by the merge launch).
 *   q_rot_out [B, Hq, d]: receives the rotated query (required).
 *   lens_next [B] int32 scratch (not used by the balanced split, which publishes the
 *     lengths from inside the decode launch).  Other arguments as llmc_rope_append /
 *     llmc_paged_decode.
 * In the fused kernel every CTA rotates its query fragments in registers and the warp
 * whose tile holds the new token rotates k and patches k/v into the landed tile and
 * the page.  Shapes the fused kernel does not take run the three separate kernels.
 */
LLMC_API int llmc_rope_append_decode(const void* q, const void* k_new, const void* v_new,
                                     void* q_rot_out, void* k_pages, void* v_pages,
                                     const int32_t* block_table, int32_t* seq_lens,
                                     const void* cos_tab, const void* sin_tab, int rope_max_pos,
                                     void* out, float* part_o, float* part_lse,
                                     int32_t* lens_next, int32_t* status, int B, int Hq, int Hkv,
                                     int d, int page_size, int max_pages_per_seq, int num_pages,
                                     int partition_tokens, float scale, int dtype,
                                     llmc_stream_t stream);

/*
 * llmc_rope_append_decode with q / k_new / v_new read in place from a wider buffer.
 * Sequence b's query is at q + b * q_seq_stride elements, with its heads d apart.
 * Its new key and value are at k_new / v_new + b * kv_seq_stride, also with heads d
 * apart. The typical source is the [B, (Hq + 2 Hkv) * d] output of a fused QKV
 * projection (attention.py:100-102 splits the same three views out of q/k/v_proj),
 * which saves three copies per layer.
 * Dense strides (Hq*d, Hkv*d) behave exactly as llmc_rope_append_decode. Other
 * strides need the fused kernel's shapes (bf16/fp16, d in {64, 128, 256}) and get
 * LLMC_EUNSUPPORTED otherwise.  flags: LLMC_DECODE_EARLY_TABLES or 0.
 */
LLMC_API int llmc_rope_append_decode_strided(
    const void* q, const void* k_new, const void* v_new, void* q_rot_out, void* k_pages,
    void* v_pages, const int32_t* block_table, int32_t* seq_lens, const void* cos_tab,
    const void* sin_tab, int rope_max_pos, void* out, float* part_o, float* part_lse,
    int32_t* lens_next, int32_t* status, int B, int Hq, int Hkv, int d, int page_size,
    int max_pages_per_seq, int num_pages, int partition_tokens, float scale, int dtype,
    long long q_seq_stride, long long kv_seq_stride, int flags, llmc_stream_t stream);

/*
 * Log-sum-exp merge of split-K partials into out [B, Hq, d].  For each (b, h)
 * with n = ceil(seq_lens[b] / partition_tokens) partitions: n >= 2 merges, n == 1
 * leaves out untouched (already written by llmc_paged_decode), n == 0 writes
 * zeros (acc / max(l, 1e-9) with an empty context, decode_attention.py:154).
 * No counterpart in the reference, which has no split-K; it completes
 * triton_decode_attention's output for long contexts.
 */
LLMC_API int llmc_lse_merge(const float* part_o, const float* part_lse, const int32_t* seq_lens, void* out,
                   int B, int Hq, int d, int max_parts, int partition_tokens, int dtype,
                   llmc_stream_t stream);

/*
 * Paged decode attention (decode + LSE merge, as llmc_paged_decode followed by
 * llmc_lse_merge) for callers that cannot allocate device memory, e.g. a host
 * framework that owns all GPU memory and gives a plugin only its input and output
 * buffers.  No counterpart in the reference.  The split-K workspace is a fixed
 * 8 MiB array inside the library (held on every GPU that loads it until exit);
 * calls needing more than llmc_paged_decode_noalloc_capacity_bytes() of partials
 * (B * Hq * max_parts * (d + 1) * 4 bytes) return LLMC_EINVAL.  The first call on a
 * device looks up the array's address; make it before any stream capture.  All calls
 * share the array, so calls that overlap on the GPU race: issue them in order on one
 * stream.  Arguments as llmc_paged_decode, minus part_o/part_lse/flags, except that
 * partition_tokens must be a positive multiple of 64: the balanced split
 * (LLMC_PARTITION_BALANCED) is not offered here and is rejected with LLMC_EINVAL.
 */
LLMC_API int llmc_paged_decode_noalloc(const void* q, const void* k_pages, const void* v_pages,
                                       const int32_t* block_table, const int32_t* seq_lens,
                                       void* out, int32_t* status, int B, int Hq, int Hkv, int d,
                                       int page_size, int max_pages_per_seq, int num_pages,
                                       int partition_tokens, float scale, int dtype,
                                       llmc_stream_t stream);

/* Bytes of the built-in scratch of llmc_paged_decode_noalloc (no counterpart in the reference). */
LLMC_API size_t llmc_paged_decode_noalloc_capacity_bytes(void);

/*
 * Decode-step helpers around the attention path (config-5 decode loop).
 *
 * llmc_add_rmsnorm: x[rows, hidden] += delta (if delta != NULL), then
 *   out = x * rsqrt(mean(x^2) + eps) * weight.  Replaces the residual add
 *   (src/llm_cuda/models/llama3/model.py:37,42) and RMSNorm.forward's torch path
 *   (src/llm_cuda/models/llama3/norm.py:31-33).
 * llmc_swiglu: out[rows, inter] = silu(g) * u with gate_up[rows, 2*inter] = [g | u].
 *   Replaces triton_swiglu's torch path (src/llm_cuda/kernels/triton/swiglu.py:103-107)
 *   on the output of a fused gate/up projection (mlp.py:39-43).
 * fp32 arithmetic, one rounding to the dtype per output.
 */
LLMC_API int llmc_add_rmsnorm(void* x, const void* delta, const void* weight, void* out, int rows,
                              int hidden, float eps, int dtype, llmc_stream_t stream);
LLMC_API int llmc_swiglu(const void* gate_up, void* out, int rows, int inter, int dtype,
                         llmc_stream_t stream);

/*
 * Decode GEMM on the tcgen05 tensor cores: y[Mb, N] = x[Mb, K] . W[N, K]^T (bf16 in,
 * fp32 accumulate in TMEM, bf16 out), Mb <= 256, N % 128 == 0, K % 64 == 0.
 * Replaces the dense projections of a decode step (nn.Linear / Column- and
 * RowParallelLinear, src/llm_cuda/parallel/tensor_parallel.py:44-49,83-90, and
 * lm_head, src/llm_cuda/models/llama3/model.py:156) at decode batch sizes, where the
 * weights are streamed once.  Persistent stream-K: every CTA takes an equal range of
 * (128-row tile, k-chunk) work; a tile shared by several CTAs is summed from their
 * fp32 parts in `workspace` (llmc_decode_gemm_workspace_bytes) by the last CTA to
 * finish, which `counters` (int32 [N / 128], all zero before the first call, left
 * zero by every call) identifies.
 */
LLMC_API size_t llmc_decode_gemm_workspace_bytes(int Mb, int N, int K);
LLMC_API int llmc_decode_gemm(const void* x, const void* w, void* y, float* workspace,
                              size_t workspace_bytes, int32_t* counters, int Mb, int N, int K,
                              int32_t* status, llmc_stream_t stream);

/* Message of the last failed call on this host thread ("" if none). */
LLMC_API const char* llmc_last_error_string(void);

/* Library version string. */
LLMC_API const char* llmc_version(void);

/*
 * Greedy pick of the decode loop: out[r] = argmax_j x[r, j] for x [rows, n] (first
 * index of the maximum; NaN counts as the maximum, as torch.argmax).  Replaces
 * torch.argmax(logits[:, -1, :], dim=-1) of src/llm_cuda/models/llama3/model.py:214.
 * workspace: llmc_argmax_workspace_bytes(rows) bytes, 8-byte aligned, zero before
 * the first call; every completed call leaves it at zero.  One launch.
 */
LLMC_API size_t llmc_argmax_workspace_bytes(int rows);
LLMC_API int llmc_argmax(const void* x, int64_t* out, int rows, int n, int dtype,
                         void* workspace, llmc_stream_t stream);

/*
 * Tensor-parallel decode: one-shot all-reduce over NVLink peer memory fused with the
 * residual add and RMSNorm.  Replaces the all-reduce of the row-parallel o_proj /
 * down_proj partials (src/llm_cuda/parallel/tensor_parallel.py:83-90) and the
 * residual add + RMSNorm after it (src/llm_cuda/models/llama3/model.py:37-42,
 * norm.py:31-33).  No counterpart in the reference, which sums the partials in one
 * process.
 *
 * Setup (once per TP group):
 *  - Every rank allocates one shared region with llmc_ipc_alloc, of
 *    llmc_ar_region_bytes bytes (zero-filled).  *flag_bytes is set to 0: the protocol
 *    needs no flag region.
 *  - The ranks exchange the llmc_ipc_handle_bytes()-byte handles, e.g. with
 *    torch.distributed.all_gather_object, and open the peers' with llmc_ipc_open.
 *  - Each rank builds a device array recv_ptrs [world]: rank q's region pointer, its
 *    own included.  flag_ptrs is not used and may be NULL.
 *  - epoch is a zeroed int32 [rows_cap] on the rank's own GPU.
 *
 * Per call, on every rank with the same rows:
 *   sum = sum over ranks of partial (fp32 in rank order, rounded to the dtype);
 *   x += sum (rounded to the dtype); out = x * rsqrt(mean(x^2) + eps) * weight.
 * One launch, one CTA per row. A row pushes its partial to every peer as 8-byte words
 * that carry 4 bytes of data and the call's epoch, and polls, bounded at 2 s, until
 * every peer's words of this epoch have arrived (no fence, no separate flag). On
 * timeout LLMC_STATUS_WAIT_TIMEOUT is set, the row is left unchanged and the row's
 * epoch still advances. The ranks' epochs may then be out of step: while the status
 * word holds that bit, calls return at once and leave their rows unchanged; stop using
 * the regions and rebuild them. Calls must be issued in the same order on all ranks.
 */
LLMC_API size_t llmc_ipc_handle_bytes(void);
LLMC_API int llmc_ipc_alloc(size_t bytes, void** dev_ptr, void* handle);
LLMC_API int llmc_ipc_open(const void* handle, void** dev_ptr);
LLMC_API int llmc_ipc_close(void* dev_ptr);
LLMC_API int llmc_ipc_free(void* dev_ptr);
LLMC_API size_t llmc_ar_region_bytes(int world, int rows_cap, int hidden, int dtype,
                                     size_t* flag_bytes);
LLMC_API int llmc_allreduce_add_rmsnorm(const void* partial, void* const* recv_ptrs,
                                        int32_t* const* flag_ptrs, int32_t* epoch, void* x,
                                        const void* weight, void* out, int32_t* status,
                                        int rank, int world, int rows, int rows_cap,
                                        int hidden, float eps, int dtype,
                                        llmc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LLM_CUDA_B200_H_ */
