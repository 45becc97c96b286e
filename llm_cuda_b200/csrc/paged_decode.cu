// Paged GQA flash-decode for sm_100a + the split-K log-sum-exp merge.
//
// Row = (sequence b, KV head, group of <= 8 query heads).  All query heads of a KV
// head (the GQA group) sit in one CTA, so every K/V byte is read from HBM once per
// step.
//
// Fast kernel (bf16/fp16, head_dim 64/128/256): persistent, one CTA per SM, 8 warps.
//  * Work split.  Balanced (partition_tokens 0, the default): the 64-token chunks of
//    all rows are laid end to end and CTA c streams chunks [c*total/G, (c+1)*total/G),
//    in pieces of <= 2048 tokens; the part of a row inside one CTA is a segment.
//    Uniform (partition_tokens T): items (row, partition of T tokens) round-robin.
//  * Warp 6, the producer, reads the block table and issues TMA (cp.async.bulk.tensor,
//    128-byte swizzle) loads of the K and V page rows of each stage into a ring of
//    shared-memory slots, signalling per-slot "full" mbarriers with transaction bytes.
//  * Warps 0-5, the consumers, in 3 groups of 2: stage s goes to group s % 3, each
//    warp of the group taking half of the stage's 16-token tiles:
//      S^T[16 tok x 8 heads] = K[16 x d] . Q^T      (mma.sync m16n8k16, K via ldmatrix)
//      online softmax per head in the log2 domain   (warp shuffles across the 8 rows)
//      O^T[d x 8 heads]     += V^T[d x 16] . P^T    (V via ldmatrix.trans, P via movmatrix)
//    then release the slot on its "empty" mbarrier.  At a segment's end the last
//    consumer warp combines the six (m, l, O) through shared memory and writes the
//    output (whole row), a partial + log2-sum-exp (uniform split), or hands the
//    partial to the merge warp (balanced split).
//  * Warp 7, the merge warp (balanced split): publishes handed-off partials, and the
//    CTA that completes a row merges it in place; it also zeroes empty rows and, in
//    the fused step, publishes the grown lengths.
//  * FUSE: RoPE of the new token's q/k and its page append happen in the same pass.
//
// Generic kernel (any dtype incl. fp32, any head_dim <= 256, any page size):
// one CTA per item, SIMT dot products, exact expf; uniform partial format.
//
// Merge kernel (uniform split): out = sum_i 2^(lse_i - M) o_i / sum_i 2^(lse_i - M).
#include <math.h>

#include <string>

#include "common.cuh"

namespace llmc {

// A context of L tokens is split into n = ceil(L / T) partitions of equal length
// (rounded up to a multiple of 64, never above T), so that the work items of one
// sequence are the same size.  Every partition is non-empty: (n-1)*len <= (n-1)*T < L.
__host__ __device__ __forceinline__ int part_len(int L, int T) {
  const int n = (L + T - 1) / T;
  return n > 0 ? ((((L + n - 1) / n) + 63) & ~63) : T;
}

// ---------------------------------------------------------------------------
// Fast kernel
// ---------------------------------------------------------------------------
namespace fast {

constexpr int kStageTok = 64;          // tokens per pipeline stage
// Consumer warps, in kGroups groups of kWarpsPerGroup.  Stage st lives in ring
// slot st % nstages and is consumed by group st % kGroups; nstages is a multiple
// of kGroups, so every slot is always consumed by the same group.  That keeps
// each mbarrier wait at most one phase behind the barrier, which parity waits
// require: were two groups to share a slot, a warp could wait on a phase parity
// that an earlier round already completed and run ahead on stale data.  Within a
// group each warp takes its own 16-token tiles of the stage and keeps its own
// softmax state; the item epilogue merges all consumer warps.
constexpr int kGroups = 3;
constexpr int kWarpsPerGroup = 2;
constexpr int kConsumers = kGroups * kWarpsPerGroup;
// Warp kConsumers is the TMA producer; warp kMergeWarp (balanced split only)
// publishes split segments and merges completed rows off the streaming path.
constexpr int kMergeWarp = kConsumers + 1;
constexpr int kThreads = (kConsumers + 2) * 32;
constexpr int kMaxStages = 12;
constexpr int kRowBytes = 128;         // one swizzle row = 64 bf16/fp16 elements

struct Params {
  const void* q;
  void* out;
  float* part_o;
  float* part_lse;
  const int32_t* block_table;
  const int32_t* seq_lens;
  int32_t* status;
  int B, Hq, Hkv, G, HG, P, max_pages, T, max_parts, num_pages, nstages;
  int max_entries;   // block-table entries one work item can touch (T / P + 2)
  float scale_log2;  // softmax scale * log2(e)
  float scale;       // softmax scale (scores are rounded as the reference's torch path)
  // Fused RoPE + append (FUSE kernels only).  q holds the RAW query; the new token of
  // sequence b sits at position seq_lens[b] (lengths before the append): its q and k
  // are rotated here with cos/sin row pos, k/v are written to the pages, and the
  // advanced lengths go to lens_next (published into seq_lens by the merge kernel).
  const void* k_new;       // [B, Hkv, D], sequence b at k_new + b * kv_stride
  const void* v_new;       // [B, Hkv, D], same strides as k_new
  const void* cos_tab;     // [rope_max_pos, D]
  const void* sin_tab;
  void* k_pages;           // pools written with the new token
  void* v_pages;
  void* q_rot_out;         // [B, Hq, D] rotated query (written once per head)
  int32_t* lens_next;      // [B]
  int rope_max_pos;
  // Balanced split (partition_tokens == 0): every CTA takes an equal contiguous range
  // of the 64-token chunks of all rows (sequence, KV head, head group) in order, cut
  // into pieces of at most cap_chunks chunks.  The part of a row that one CTA covers
  // is a segment: its partial goes to slot (row + CTA index), unique over all
  // segments.  The CTA that completes a row's last segment merges the row
  // (counters[row] counts finished segments); counters[rows] counts CTAs past their
  // length reads, and the last of them publishes the grown lengths (FUSE).  Every
  // counter is returned to zero by the CTA that completes it.
  int balanced;
  int cap_chunks;
  int32_t* counters;       // [rows + 1], zero between calls
  long long q_stride;      // elements between the queries of consecutive sequences
  long long kv_stride;     // the same for k_new / v_new (heads are D apart in both)
  int32_t* seq_lens_out;   // FUSE + balanced: lengths after the step are written here
  // Balanced split only: seq_lens, the block table and the page pools are not written
  // by any kernel that can still be running when this one starts, so the length scan,
  // the work split and the K/V stream begin before griddepcontrol.wait; only the
  // roles that read the previous kernel's output (q, new k/v) or write anything wait.
  int early;
};

// Byte offset of (row, 16-byte chunk) inside a 128B-swizzled region whose base is
// 1024-byte aligned (TMA SWIZZLE_128B: chunk index XOR row % 8).
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return row * kRowBytes + ((chunk ^ (row & 7)) << 4);
}

struct Item {
  int b, part, kvh, hg, t0, t1, L;
};

// Work item i -> (sequence, partition, KV head, head group).  Reads only shared
// memory: the item prefix sums and the (clamped) sequence lengths.
__device__ __forceinline__ Item decode_item(int i, const int* prefix, int B, int Hkv, int HG,
                                            const int* lens, int T) {
  // prefix[b] = number of items before sequence b; binary search for b.
  int lo = 0, hi = B;  // prefix[lo] <= i < prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (prefix[mid] <= i) lo = mid; else hi = mid;
  }
  Item it;
  it.b = lo;
  const int r = i - prefix[lo];
  const int per_part = Hkv * HG;
  it.part = r / per_part;
  const int kh = r - it.part * per_part;
  it.kvh = kh / HG;
  it.hg = kh - it.kvh * HG;
  it.L = lens[it.b];
  const int plen = part_len(it.L, T);
  it.t0 = it.part * plen;
  it.t1 = min(it.L, it.t0 + plen);
  return it;
}

// A piece: consecutive stages of one row that a CTA processes without a break.
// first/last: the piece opens/closes this CTA's segment of the row (softmax state
// is reset before the first and written out after the last); whole: the segment is
// the entire row, so the result goes straight to `out`.  part: uniform mode, the
// partition index; balanced mode, the partial slot.
struct Piece {
  int b, kvh, hg, t0, t1, L, part;
  bool first, last, whole;
  // Balanced, last piece of a split row's segment: CTAs cf..cl hold the row (nlive
  // of them own chunks); total = chunks of all rows.
  int cf, cl, nlive;
  int total;
};

// The split of `total` chunks (< 2^31) into G ranges [start(c), start(c+1)) with
// start(c) = floor(c * total / G), in 32-bit arithmetic: with total = q*G + r,
// start(c) = c*q + floor(c*r / G) exactly (c*q < 2^31, c*r < G^2).  64-bit integer
// division is a long software routine on the GPU; this runs in a few instructions.
struct ChunkSplit {
  int q, r, G, total;
  __device__ __forceinline__ void init(int total_, int G_) {
    total = total_; G = G_; q = total_ / G_; r = total_ - q * G_;
  }
  __device__ __forceinline__ int start(int c) const { return c * q + (c * r) / G; }
  // CTA owning chunk x (0 <= x < total): the largest c with start(c) <= x.  A float
  // estimate is within one of it; the exact starts settle the rest.
  __device__ __forceinline__ int owner(int x) const {
    int c = (int)((float)x * (float)G / (float)total);
    c = c < 0 ? 0 : (c >= G ? G - 1 : c);
    while (c + 1 < G && start(c + 1) <= x) ++c;
    while (c > 0 && start(c) > x) --c;
    return c;
  }
  __device__ __forceinline__ bool live(int c) const { return start(c) != start(c + 1); }
};

// The sequence of pieces of this CTA.  Uniform mode: items blockIdx.x, +gridDim.x,
// ... (one piece each).  Balanced mode: a walk over chunks [start, end) of the
// flattened row space; prefix[] holds per-sequence chunk prefix sums and every row
// of sequence b has prefix[b+1] - prefix[b] chunks.
struct Walker {
  const int* prefix;
  const int* lens;
  int B, Hkv, HG, T, cap, total_items;
  bool balanced;
  int i, phase;
  // Chunk positions in the flattened row space; the host keeps the total below 2^31.
  int x, start, end, p0, phase_end;
  ChunkSplit split;

  // Sequence b of flattened chunk x and the first chunk of x's row.
  __device__ void locate(int xx, int& b, int& row_begin) const {
    const int RS = Hkv * HG;
    const int key = xx / RS;             // prefix[b] * RS <= xx  <=>  prefix[b] <= xx / RS
    int lo = 0, hi = B;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (prefix[mid] <= key) lo = mid; else hi = mid;
    }
    b = lo;
    const int n = prefix[b + 1] - prefix[b];
    const int local = xx - prefix[b] * RS;
    row_begin = xx - local % n;
  }

  __device__ void init(const Params& p, const int* pre, const int* ln) {
    prefix = pre; lens = ln; B = p.B; Hkv = p.Hkv; HG = p.HG; T = p.T; cap = p.cap_chunks;
    balanced = p.balanced != 0;
    total_items = prefix[B];
    i = blockIdx.x;
    split.init(prefix[B] * Hkv * HG, gridDim.x);
    start = split.start(blockIdx.x);
    end = split.start(blockIdx.x + 1);
    // The range's last segment (usually the head of a row that the next CTA
    // continues) goes first, then the range from its start: both segments a CTA
    // shares with its neighbours finish early, so the row merges they trigger run
    // while the other CTAs are still streaming rather than at the end.
    p0 = start;
    if (balanced && end > start) {
      int b, rb;
      locate(end - 1, b, rb);
      p0 = rb > start ? rb : start;
    }
    phase = 0;
    x = p0;
    phase_end = end;
  }

  __device__ bool next(Piece& pc) {
    if (!balanced) {
      if (i >= total_items) return false;
      const Item it = decode_item(i, prefix, B, Hkv, HG, lens, T);
      i += gridDim.x;
      pc.b = it.b; pc.kvh = it.kvh; pc.hg = it.hg; pc.t0 = it.t0; pc.t1 = it.t1;
      pc.L = it.L; pc.part = it.part;
      pc.first = pc.last = true;
      pc.whole = it.L <= T;
      pc.cf = pc.cl = pc.nlive = 0;
      pc.total = 0;
      return true;
    }
    if (x >= phase_end) {
      if (phase == 1 || p0 == start) return false;
      phase = 1;
      x = start;
      phase_end = p0;
    }
    const int RS = Hkv * HG;
    int b, row_begin;
    locate(x, b, row_begin);
    const int n = prefix[b + 1] - prefix[b];
    const int ri = (row_begin - prefix[b] * RS) / n;
    const int c0 = x - row_begin;
    const int row_end = row_begin + n;
    int e = phase_end < row_end ? phase_end : row_end;
    if (e > x + cap) e = x + cap;
    pc.b = b; pc.kvh = ri / HG; pc.hg = ri - pc.kvh * HG;
    pc.L = lens[b];
    pc.t0 = c0 * kStageTok;
    pc.t1 = min(pc.L, (int)((c0 + (e - x)) * kStageTok));
    pc.first = x == (row_begin > start ? row_begin : start);
    pc.last = e == (row_end < end ? row_end : end);
    pc.whole = row_begin >= start && row_end <= end;
    pc.part = (b * Hkv + pc.kvh) * HG + pc.hg + blockIdx.x;
    pc.cf = pc.cl = pc.nlive = 0;
    pc.total = 0;
    if (!pc.whole && pc.last) {   // only the segment epilogue needs them
      pc.total = split.total;
      pc.cf = split.owner(row_begin);
      pc.cl = split.owner(row_end - 1);
      if (split.total >= split.G) {
        pc.nlive = pc.cl - pc.cf + 1;
      } else {   // some CTAs own no chunk and hold no segment
        for (int c = pc.cf; c <= pc.cl; ++c) pc.nlive += split.live(c);
      }
    }
    x = e;
    return true;
  }
};

// Log-sum-exp merge of one row's segment partials, by one warp: lane = (head hn,
// quarter dq of head_dim).  out = sum_c 2^(lse_c - M) o_c / sum_c 2^(lse_c - M) over
// the CTAs c in [cf, cl] that own chunks.  Partials of other CTAs are read through
// L2 (ld.global.cg), so no stale L1 line is used.
template <int D, typename T>
__device__ __forceinline__ void merge_row(const Params& p, const Piece& it, int r, int hn, int dq,
                                          int nh) {
  if (hn >= nh) return;
  const int G = gridDim.x;
  ChunkSplit split;
  split.init(it.total, G);
  auto live = [&](int cc) -> bool { return cc <= it.cl && (it.total >= G || split.live(cc)); };
  const float* lse = p.part_lse + (size_t)r * 8 + hn;
  const float* pobase = p.part_o + ((size_t)r * 8 + hn) * D + dq;
  const int hq = it.kvh * p.G + it.hg * 8 + hn;
  T* orow = reinterpret_cast<T*>(p.out) + ((size_t)it.b * p.Hq + hq) * D + dq;
  constexpr int U = 4;                       // segments whose loads are issued together
  if (D <= 128 && it.cl - it.cf < U) {
    // At most 4 CTAs hold the row (the usual case): every log2-sum-exp and every
    // partial value of this lane is requested at once, one L2 round trip in all.
    constexpr int DL = D / 4;
    float l[U], v[U][DL];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool ok = live(it.cf + u);
      l[u] = ok ? __ldcg(lse + (size_t)(it.cf + u) * 8) : -INFINITY;
      const float* po = pobase + (size_t)(it.cf + u) * 8 * D;
#pragma unroll
      for (int j = 0; j < DL; ++j) v[u][j] = ok ? __ldcg(po + 4 * j) : 0.f;
    }
    float M = l[0];
#pragma unroll
    for (int u = 1; u < U; ++u) M = fmaxf(M, l[u]);
    float w[U], S = 0.f;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      w[u] = exp2f(l[u] - M);
      S += w[u];
    }
    const float inv = 1.f / S;
#pragma unroll
    for (int j = 0; j < DL; ++j) {
      float a = 0.f;
#pragma unroll
      for (int u = 0; u < U; ++u) a = fmaf(w[u], v[u][j], a);
      orow[4 * j] = from_f32<T>(a * inv);
    }
    return;
  }
  constexpr int DPL = D / 4;                 // head_dim values of this lane: dq + 4j
  constexpr int CH = DPL < 16 ? DPL : 16;    // accumulated per pass
  // Online max / sum over the segments' log2-sum-exps, U loads in flight at a time.
  float M = -INFINITY, S = 0.f;
  float l0[U];
  for (int c0 = it.cf; c0 <= it.cl; c0 += U) {
    float l[U];
#pragma unroll
    for (int u = 0; u < U; ++u) l[u] = live(c0 + u) ? __ldcg(lse + (size_t)(c0 + u) * 8) : -INFINITY;
    float mb = M;
#pragma unroll
    for (int u = 0; u < U; ++u) mb = fmaxf(mb, l[u]);
    S *= exp2f(M - mb);                      // M = -inf on the first batch: S = 0 anyway
#pragma unroll
    for (int u = 0; u < U; ++u) S += exp2f(l[u] - mb);
    M = mb;
    if (c0 == it.cf) {
#pragma unroll
      for (int u = 0; u < U; ++u) l0[u] = l[u];
    }
  }
  const float inv = 1.f / S;
  const bool one_batch = it.cl - it.cf < U;  // weights straight from registers
#pragma unroll 1
  for (int j0 = 0; j0 < DPL; j0 += CH) {
    float acc[CH];
#pragma unroll
    for (int j = 0; j < CH; ++j) acc[j] = 0.f;
    for (int c0 = it.cf; c0 <= it.cl; c0 += U) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cc = c0 + u;
        if (!live(cc)) continue;
        const float lv = one_batch ? l0[u] : __ldcg(lse + (size_t)cc * 8);
        const float w = exp2f(lv - M) * inv;
        const float* po = pobase + (size_t)cc * 8 * D + 4 * j0;
#pragma unroll
        for (int j = 0; j < CH; ++j) acc[j] = fmaf(w, __ldcg(po + 4 * j), acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < CH; ++j) orow[4 * (j0 + j)] = from_f32<T>(acc[j]);
  }
}

template <int D, typename T, int ST, bool FUSE>
__global__ void __launch_bounds__(kThreads, 1)
paged_decode_tma_kernel(const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const Params p) {
  constexpr int HALVES = D / 64;
  constexpr int KC = D / 16;                    // k-chunks of 16 along head_dim
  constexpr int HALF_BYTES = ST * kRowBytes;          // 8 KB
  constexpr int KV_BYTES = HALVES * HALF_BYTES;              // K (or V) of one stage
  constexpr int STAGE_BYTES = 2 * KV_BYTES;
  // d = 128: one 3-D TMA box {64 cols, 2 halves, rows} brings a whole (page, head)
  // chunk, landing as [token][half][64] (swizzle row = 2*token + half).  Other head
  // dims use one 2-D box per 64-column half, landing as [half][token][64].
  constexpr bool kInterleave = (D == 128);
  auto smem_off = [](int tok, int d0) -> uint32_t {
    return kInterleave ? swz(tok * 2 + (d0 >> 6), (d0 & 63) >> 3)
                       : (d0 >> 6) * HALF_BYTES + swz(tok, (d0 & 63) >> 3);
  };

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
  const int nst = p.nstages;
  uint8_t* ring = smem;
  float* comb_o = reinterpret_cast<float*>(smem + nst * STAGE_BYTES);  // [kConsumers][D][8]
  float* comb_m = comb_o + kConsumers * D * 8;                        // [kConsumers][8]
  float* comb_l = comb_m + kConsumers * 8;                            // [kConsumers][8]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(comb_l + kConsumers * 8);
  uint64_t* empty_bar = full_bar + kMaxStages;
  int* prefix = reinterpret_cast<int*>(empty_bar + kMaxStages);       // [B + 1]
  int* lens = prefix + p.B + 1;                                        // [B]
  int* bt_s = lens + p.B;                                              // [2][max_entries]
  volatile int* abort_flag = bt_s + 2 * p.max_entries;
  int* comb_count = bt_s + 2 * p.max_entries + 1;        // warps done with the current item
  volatile int* comb_done = bt_s + 2 * p.max_entries + 2; // items combined so far
  volatile int* pend_flag = bt_s + 2 * p.max_entries + 3; // handoff slot: 1 = holds a segment
  // Handoff slot of a split segment's combined partial, consumers -> merge warp:
  // normalised o [8 heads][D] then log2-sum-exp [8].
  float* pend_o = reinterpret_cast<float*>(bt_s + 2 * p.max_entries + 4);
  float* pend_lse = pend_o + 8 * D;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- set-up: barriers + per-sequence item prefix sums (producer warp scans) ----
  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kWarpsPerGroup);
    }
    *abort_flag = 0;
    *comb_count = 0;
    *comb_done = 0;
    *pend_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kConsumers && lane == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
  }
  if (warp == kConsumers && lane == 1) {
    // The block table is read right after the length scan; by then the previous
    // step's K/V stream has evicted it from L2.  Each CTA asks L2 for its share now,
    // overlapping the previous kernel (a hint only: the reads that matter come after
    // griddepcontrol.wait, and L2 is coherent with any write to the table before it).
    const uintptr_t base = reinterpret_cast<uintptr_t>(p.block_table);
    const size_t bytes = (size_t)p.B * p.max_pages * sizeof(int32_t);
    const size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
    const size_t off = per * blockIdx.x;
    if ((base & 15) == 0 && off < bytes) {
      const size_t n = (bytes - off < per ? bytes - off : per) & ~(size_t)15;
      if (n)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off),
                     "r"((uint32_t)n)
                     : "memory");
    }
  }
  // Everything above overlaps the previous kernel under programmatic dependent
  // launch; lengths, block table and pages are read only after this wait, unless the
  // caller vouched for them (p.early), in which case the consumer and merge warps wait
  // below, before their first read of the previous kernel's output or first write.
  if (!p.early) pdl_wait();
  pdl_launch_dependents();
  if (warp == kConsumers) {
    const int per = (p.B + 31) / 32;
    const int lo = min(p.B, lane * per), hi = min(p.B, lo + per);
    const int per_part = p.Hkv * p.HG;
    int sum = 0;
    // Tokens attended by sequence b: its length, plus the new token when fused.
    auto eff_len = [&](int b, bool report) -> int {
      int L = p.seq_lens[b] + (FUSE ? 1 : 0);
      const int cap = p.max_pages * p.P;
      if (L > cap) {
        if (report) atomicOr(p.status, FUSE ? kStatusAppendOverflow : kStatusSeqLenRange);
        L = cap;
      }
      if (FUSE && report && L > p.rope_max_pos) atomicOr(p.status, kStatusRopeRange);
      return L;
    };
    // Work units of sequence b: uniform mode, its items; balanced mode, the 64-token
    // chunks of one of its rows.
    auto units = [&](int L) -> int {
      if (L <= 0) return 0;
      return p.balanced ? (L + kStageTok - 1) / kStageTok : (L + p.T - 1) / p.T * per_part;
    };
    for (int b = lo; b < hi; ++b) sum += units(eff_len(b, true));
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - sum;
    for (int b = lo; b < hi; ++b) {
      prefix[b] = run;
      const int L = eff_len(b, false);
      lens[b] = L;
      if (FUSE && !p.balanced && blockIdx.x == 0) p.lens_next[b] = L;   // for the merge launch
      run += units(L);
    }
    if (lane == 31) prefix[p.B] = incl;
  }
  __syncthreads();

  if (warp == kMergeWarp) {
    // ======================= merge warp =======================
    if (!p.balanced) return;
    if (p.early) pdl_wait();
    const int n_rows = p.B * p.Hkv * p.HG;
    // Empty contexts have no chunk: their rows get acc / max(l, 1e-9) = 0 here.
    for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
      if (lens[b] != 0) continue;
      T* ob = reinterpret_cast<T*>(p.out) + (size_t)b * p.Hq * D;
      for (int i = lane; i < p.Hq * D; i += 32) ob[i] = from_f32<T>(0.f);
    }
    if (FUSE) {
      // Every CTA has read seq_lens (before the barrier above); the last one to get
      // here publishes the grown lengths and re-arms the counter.
      int last = 0;
      if (lane == 0) last = atomicAdd(&p.counters[n_rows], 1) == (int)gridDim.x - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        for (int b = lane; b < p.B; b += 32) p.seq_lens_out[b] = lens[b];
        if (lane == 0) p.counters[n_rows] = 0;
      }
    }
    // Split segments arrive through the handoff slot in walk order.
    const int hn = lane & 7, dq = lane >> 3;
    Walker walk;
    walk.init(p, prefix, lens);
    Piece it;
    while (walk.next(it)) {
      if (!it.last || it.whole) continue;
      {
        const unsigned long long t0 = globaltimer_ns();
        while (*pend_flag == 0 && !*abort_flag) {
          if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            *abort_flag = 1;
            atomicOr(p.status, kStatusWaitTimeout);
          }
        }
      }
      if (*abort_flag) break;
      __threadfence_block();
      const int nh = min(8, p.G - it.hg * 8);
      const size_t pidx = (size_t)it.part * 8 + hn;
      if (hn < nh) {
        for (int d = dq; d < D; d += 4) p.part_o[pidx * D + d] = pend_o[hn * D + d];
        if (dq == 0) p.part_lse[pidx] = pend_lse[hn];
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) *pend_flag = 0;            // the slot has been read
      const int r = (it.b * p.Hkv + it.kvh) * p.HG + it.hg;
      __threadfence();
      int done = 0;
      if (lane == 0) done = atomicAdd(&p.counters[r], 1) == it.nlive - 1;
      done = __shfl_sync(0xffffffffu, done, 0);
      if (done) {
        __threadfence();
        merge_row<D, T>(p, it, r, hn, dq, nh);
        __syncwarp();
        if (lane == 0) p.counters[r] = 0;
      }
    }
    return;
  }

  if (warp == kConsumers) {
    // ======================= producer warp =======================
    // The block-table slice of the NEXT item is prefetched with cp.async into the
    // other half of a double buffer while the current item's stages are issued,
    // so no stage waits on a dependent global load.
    uint32_t stage = 0;
    auto prefetch_bt = [&](const Piece& it, int buf) {
      const int32_t* row = p.block_table + (size_t)it.b * p.max_pages;
      const int first = it.t0 / p.P;
      const int n = (it.t1 - 1) / p.P - first + 1;
      const uint32_t dst = smem_u32(bt_s + buf * p.max_entries);
      for (int e = lane; e < n; e += 32) cp_async_4(dst + 4 * e, row + first + e);
      cp_async_commit();
    };
    int buf = 0;
    Walker walk;
    walk.init(p, prefix, lens);
    Piece it{};
    bool has = walk.next(it);
    if (has) prefetch_bt(it, 0);
    for (; has; buf ^= 1) {
      Piece nx{};
      const bool has_next = walk.next(nx);
      if (has_next) {
        prefetch_bt(nx, buf ^ 1);
        cp_async_wait<1>();      // this item's slice has landed (the next may be in flight)
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();
      const int* ids = bt_s + buf * p.max_entries;
      const int item_first = it.t0 / p.P;
      const int nstage = (it.t1 - it.t0 + ST - 1) / ST;
      for (int s = 0; s < nstage; ++s, ++stage) {
        const int slot = stage % nst;
        const uint32_t round = stage / nst;
        const int tok0 = it.t0 + s * ST;
        // Pages touched by this stage and the box (rows) loaded from each.
        int npg, rows, first_page, row0;
        if (p.P >= ST) {
          npg = 1; rows = ST; first_page = tok0 / p.P; row0 = tok0 - first_page * p.P;
        } else {
          first_page = tok0 / p.P; row0 = 0; rows = p.P;
          npg = min(ST / p.P, (it.t1 - first_page * p.P + p.P - 1) / p.P);
        }
        // Lane j < npg takes page id j of this stage.
        int page = 0;
        bool page_ok = true;
        if (lane < npg) {
          page = ids[first_page - item_first + lane];
          if (page < 0 || page >= p.num_pages) {
            atomicOr(p.status, kStatusBadPage);
            page_ok = false;
          }
        }
        const unsigned okmask = __ballot_sync(0xffffffffu, lane < npg && page_ok);
        const uint32_t bytes = __popc(okmask) * 2u * HALVES * rows * kRowBytes;  // K + V
        const uint32_t fb = smem_u32(&full_bar[slot]);
        mbar_wait_bounded(smem_u32(&empty_bar[slot]), (round & 1u) ^ 1u, abort_flag, p.status);
        if (lane == 0) mbar_arrive_expect_tx(fb, bytes);
        __syncwarp();
        if (!*abort_flag && lane < npg && page_ok) {
          const int row = (page * p.Hkv + it.kvh) * p.P + row0;
          const uint32_t sbase = smem_u32(ring + slot * STAGE_BYTES);
          if constexpr (kInterleave) {
            const uint32_t kdst = sbase + lane * rows * HALVES * kRowBytes;
            tma_load_3d(kdst, &tmap_k, 0, 0, row, fb);
            tma_load_3d(kdst + KV_BYTES, &tmap_v, 0, 0, row, fb);
          } else {
            const uint32_t kdst = sbase + lane * rows * kRowBytes;
#pragma unroll
            for (int h = 0; h < HALVES; ++h) {
              tma_load_2d(kdst + h * HALF_BYTES, &tmap_k, h * 64, row, fb);
              tma_load_2d(kdst + KV_BYTES + h * HALF_BYTES, &tmap_v, h * 64, row, fb);
            }
          }
        }
      }
      __syncwarp();   // all lanes done with this buffer before it is refilled
      it = nx;
      has = has_next;
    }
    // Drain: wait (bounded) for the last load issued into every slot.
    if (lane == 0) {
      const uint32_t n = stage < (uint32_t)nst ? stage : (uint32_t)nst;
      for (uint32_t k = 0; k < n; ++k) {
        const uint32_t st = stage - 1 - k;
        mbar_wait_bounded(smem_u32(&full_bar[st % nst]), (st / nst) & 1u, abort_flag, p.status);
      }
    }
    return;
  }

  // ======================= consumer warps =======================
  if (p.early) pdl_wait();   // q, the new token's k/v, and every write come after it
  const int g = lane >> 2;   // fragment row group
  const int c = lane & 3;    // fragment column pair
  const T* qbase = reinterpret_cast<const T*>(p.q);
  uint32_t stage = 0;

  // Q^T as the B operand (k = head_dim, n = head): b0b1 = q[n][16kc+2c..], b2b3 = +8.
  // The next item's fragments are loaded while the current item runs.
  // With FUSE the cos/sin pairs of the fragment's first-half columns at the new
  // token's position come along; the rotation happens when the item starts.
  constexpr int KH = KC / 2;            // k-chunks in the first half of head_dim
  auto load_q = [&](const Piece& it, uint32_t (&dst)[KC][2], uint32_t (&cs)[KH][2],
                    uint32_t (&sn)[KH][2]) {
    const int ghead = it.hg * 8 + g;
    const bool ok = ghead < p.G;
    const T* qrow = qbase + (size_t)it.b * p.q_stride + (size_t)(ok ? it.kvh * p.G + ghead : 0) * D;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      dst[kc][0] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kc * 16 + 2 * c)) : 0u;
      dst[kc][1] = ok ? __ldg(reinterpret_cast<const uint32_t*>(qrow + kc * 16 + 2 * c + 8)) : 0u;
    }
    if constexpr (FUSE) {
      const int pos = max(it.L - 1, 0);
      const T* crow = reinterpret_cast<const T*>(p.cos_tab) + (size_t)pos * D;
      const T* srow = reinterpret_cast<const T*>(p.sin_tab) + (size_t)pos * D;
#pragma unroll
      for (int kc = 0; kc < KH; ++kc)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          cs[kc][r] = __ldg(reinterpret_cast<const uint32_t*>(crow + kc * 16 + 2 * c + 8 * r));
          sn[kc][r] = __ldg(reinterpret_cast<const uint32_t*>(srow + kc * 16 + 2 * c + 8 * r));
        }
    }
  };
  constexpr int NT = ST / 16;                 // 16-token tiles per stage
  constexpr int NTL = NT / kWarpsPerGroup;    // tiles of this warp
  const int sub = warp % kWarpsPerGroup;
  // FUSE: the new token's raw k/v, cos/sin and page id, fetched one piece ahead by
  // the warp whose tile will hold the token, so that patching it into the landed
  // tile costs no global round trip on the streaming path.  Lane j holds elements
  // i = 2j + 64n of each half of head_dim.
  constexpr int NI = (D / 2 + 63) / 64;
  struct NewTok {
    uint32_t k1[NI], k2[NI], v1[NI], v2[NI], cs[NI], sn[NI];
    int page;
  };
  auto fetch_newtok = [&](const Piece& x, NewTok& nt) {
    const int pos = x.L - 1;
    const T* kn = reinterpret_cast<const T*>(p.k_new) + (size_t)x.b * p.kv_stride + (size_t)x.kvh * D;
    const T* vn = reinterpret_cast<const T*>(p.v_new) + (size_t)x.b * p.kv_stride + (size_t)x.kvh * D;
    const T* crow = reinterpret_cast<const T*>(p.cos_tab) + (size_t)pos * D;
    const T* srow = reinterpret_cast<const T*>(p.sin_tab) + (size_t)pos * D;
    nt.page = __ldg(p.block_table + (size_t)x.b * p.max_pages + pos / p.P);
#pragma unroll
    for (int n = 0; n < NI; ++n) {
      const int i = 2 * lane + 64 * n;
      if (i < D / 2) {
        nt.k1[n] = __ldg(reinterpret_cast<const uint32_t*>(kn + i));
        nt.k2[n] = __ldg(reinterpret_cast<const uint32_t*>(kn + i + D / 2));
        nt.v1[n] = __ldg(reinterpret_cast<const uint32_t*>(vn + i));
        nt.v2[n] = __ldg(reinterpret_cast<const uint32_t*>(vn + i + D / 2));
        nt.cs[n] = __ldg(reinterpret_cast<const uint32_t*>(crow + i));
        nt.sn[n] = __ldg(reinterpret_cast<const uint32_t*>(srow + i));
      }
    }
  };
  // Does this warp patch the new token of piece x, whose first stage is stage0?
  auto owns_newtok = [&](const Piece& x, uint32_t stage0) -> bool {
    const int pos = x.L - 1;
    if (!FUSE || pos < x.t0 || pos >= x.t1) return false;
    const int s_new = (pos - x.t0) / ST;
    if ((int)((stage0 + s_new) % kGroups) != warp / kWarpsPerGroup) return false;
    return (pos - x.t0 - s_new * ST) / (NTL * 16) == sub;
  };
  NewTok nt_next;
  bool nt_next_ok = false;

  uint32_t qf_next[KC][2];
  uint32_t cs_next[KH][2], sn_next[KH][2];
  Walker walk;
  walk.init(p, prefix, lens);
  Piece it_next{};
  bool has = walk.next(it_next);
  if (has) load_q(it_next, qf_next, cs_next, sn_next);
  if (has && owns_newtok(it_next, 0)) {
    fetch_newtok(it_next, nt_next);
    nt_next_ok = true;
  }
  int item_seq = 0;   // segments this CTA has finished
  uint32_t qf[KC][2];
  float m_run[2] = {-INFINITY, -INFINITY};   // heads 2c, 2c+1 (log2 domain)
  float l_run[2] = {0.f, 0.f};               // per-thread partial sums
  float o[KC][4];                            // O^T fragments: rows d, cols heads
  while (has) {
    const Piece it = it_next;
    if (it.first) {
#pragma unroll
      for (int kc = 0; kc < KC; ++kc) {
        qf[kc][0] = qf_next[kc][0];
        qf[kc][1] = qf_next[kc][1];
      }
    }
    if (FUSE && it.first) {
      // RoPE of the new token's query, in registers: element d of the first half
      // (chunk kc) pairs with d + D/2 (chunk kc + KC/2) held by the same lane.
#pragma unroll
      for (int kc = 0; kc < KH; ++kc)
#pragma unroll
        for (int r = 0; r < 2; ++r) rope_pair2<T>(qf[kc][r], qf[kc + KH][r], cs_next[kc][r], sn_next[kc][r]);
      // The partition-0 item of each head group publishes the rotated query.
      const int ghead = it.hg * 8 + g;
      if (p.q_rot_out != nullptr && it.t0 == 0 && warp == 0 && ghead < p.G) {
        uint32_t* qo = reinterpret_cast<uint32_t*>(
            reinterpret_cast<T*>(p.q_rot_out) + ((size_t)it.b * p.Hq + it.kvh * p.G + ghead) * D);
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
          qo[(kc * 16 + 2 * c) / 2] = qf[kc][0];
          qo[(kc * 16 + 2 * c + 8) / 2] = qf[kc][1];
        }
      }
    }
    NewTok nt = nt_next;
    bool nt_ok = nt_next_ok;
    const int nstage = (it.t1 - it.t0 + ST - 1) / ST;
    has = walk.next(it_next);
    if (has && it_next.first) load_q(it_next, qf_next, cs_next, sn_next);
    nt_next_ok = false;
    if (has && owns_newtok(it_next, stage + nstage)) {
      fetch_newtok(it_next, nt_next);
      nt_next_ok = true;
    }
    if (it.first) {
      m_run[0] = m_run[1] = -INFINITY;
      l_run[0] = l_run[1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KC; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }

    for (int s = 0; s < nstage; ++s, ++stage) {
      if ((int)(stage % kGroups) != warp / kWarpsPerGroup) continue;
      const int slot = stage % nst;
      const uint32_t round = stage / nst;
      mbar_wait_bounded(smem_u32(&full_bar[slot]), round & 1u, abort_flag, p.status);
      const int tok0 = it.t0 + s * ST;
      const int nvalid = min(ST, it.t1 - tok0);
      const int row_lo = sub * NTL * 16;               // this warp's token rows
      const int my_valid = min(max(nvalid - row_lo, 0), NTL * 16);
      const int my_tiles = (my_valid + 15) >> 4;
      uint8_t* kst = ring + slot * STAGE_BYTES;
      uint8_t* vst = kst + KV_BYTES;
      bool patched = false;
      if constexpr (FUSE) {
        // The new token lands in this warp's rows: its page slot was never written, so
        // put the rotated k row and the v row straight into the landed tile, and into
        // the page for later steps (one head group per KV head writes the page).
        const int pos = it.L - 1;
        const int r = pos - tok0;
        if (r >= row_lo && r < row_lo + my_valid) {
          if (!nt_ok) fetch_newtok(it, nt);   // not prefetched (not expected): fetch now
          const int page = nt.page;
          const bool write_page = it.hg == 0 && page >= 0 && page < p.num_pages;
          T* kp = reinterpret_cast<T*>(p.k_pages) +
                  (((size_t)(write_page ? page : 0) * p.Hkv + it.kvh) * p.P + pos % p.P) * D;
          T* vp = reinterpret_cast<T*>(p.v_pages) + (kp - reinterpret_cast<T*>(p.k_pages));
#pragma unroll
          for (int n = 0; n < NI; ++n) {
            const int i = 2 * lane + 64 * n;
            if (i >= D / 2) continue;
            uint32_t x1 = nt.k1[n];
            uint32_t x2 = nt.k2[n];
            rope_pair2<T>(x1, x2, nt.cs[n], nt.sn[n]);
            const uint32_t v1 = nt.v1[n];
            const uint32_t v2 = nt.v2[n];
            *reinterpret_cast<uint32_t*>(kst + smem_off(r, i) + (i & 7) * 2) = x1;
            *reinterpret_cast<uint32_t*>(kst + smem_off(r, i + D / 2) + (i & 7) * 2) = x2;
            *reinterpret_cast<uint32_t*>(vst + smem_off(r, i) + (i & 7) * 2) = v1;
            *reinterpret_cast<uint32_t*>(vst + smem_off(r, i + D / 2) + (i & 7) * 2) = v2;
            if (write_page) {
              *reinterpret_cast<uint32_t*>(kp + i) = x1;
              *reinterpret_cast<uint32_t*>(kp + i + D / 2) = x2;
              *reinterpret_cast<uint32_t*>(vp + i) = v1;
              *reinterpret_cast<uint32_t*>(vp + i + D / 2) = v2;
            }
          }
          patched = true;
          __syncwarp();
        }
      }
      if (my_tiles > 0) {
        if (my_valid < my_tiles * 16) {
          // Rows past the context may hold stale or never-written bytes (possibly
          // NaN); probabilities there are 0 but 0*NaN is NaN, so zero the V rows
          // of this warp's last tile beyond the context.
          const int r0 = row_lo + my_valid, r1 = row_lo + my_tiles * 16;
          const int nchunk = (r1 - r0) * 8;
          if constexpr (kInterleave) {
            for (int k = lane; k < nchunk * HALVES; k += 32)
              *reinterpret_cast<uint4*>(vst + r0 * HALVES * kRowBytes + k * 16) =
                  make_uint4(0, 0, 0, 0);
          } else {
#pragma unroll
            for (int h = 0; h < HALVES; ++h)
              for (int k = lane; k < nchunk; k += 32)
                *reinterpret_cast<uint4*>(vst + h * HALF_BYTES + r0 * kRowBytes + k * 16) =
                    make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        const uint32_t kaddr = smem_u32(kst);
        const uint32_t vaddr = smem_u32(vst);

        // ---- S^T = K . Q^T for this warp's tiles (kc outer: independent chains) ----
        // Two accumulators per tile (even / odd k-chunks) halve the dependent mma chain.
        float sacc[NTL][4], sacc2[NTL][4];
#pragma unroll
        for (int j = 0; j < NTL; ++j)
#pragma unroll
          for (int r = 0; r < 4; ++r) sacc[j][r] = sacc2[j][r] = 0.f;
#pragma unroll
        for (int kc = 0; kc < KC; ++kc) {
          const int d0 = kc * 16 + (lane >> 4) * 8;
#pragma unroll
          for (int j = 0; j < NTL; ++j) {
            if (j < my_tiles) {
              const int row = row_lo + j * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
              uint32_t a[4];
              ldsm_x4(kaddr + smem_off(row, d0), a[0], a[1], a[2], a[3]);
              Mma<T>::run((kc & 1) ? sacc2[j] : sacc[j], a, qf[kc][0], qf[kc][1]);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < NTL; ++j)
#pragma unroll
          for (int r = 0; r < 4; ++r) sacc[j][r] += sacc2[j][r];
        // ---- online softmax (log2 domain); c0/c2 -> head 2c, c1/c3 -> head 2c+1 ----
        float mloc[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int j = 0; j < NTL; ++j) {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int tok = j * 16 + g + ((r >> 1) << 3);
            // scores rounded at the reference torch path's points, then log2 domain
            const float v = (tok < my_valid)
                                ? ref_score<T>(sacc[j][r], p.scale) * 1.4426950408889634f
                                : -INFINITY;
            sacc[j][r] = v;
            mloc[r & 1] = fmaxf(mloc[r & 1], v);
          }
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          mloc[j] = fmaxf(mloc[j], __shfl_xor_sync(0xffffffffu, mloc[j], 4));
          mloc[j] = fmaxf(mloc[j], __shfl_xor_sync(0xffffffffu, mloc[j], 8));
          mloc[j] = fmaxf(mloc[j], __shfl_xor_sync(0xffffffffu, mloc[j], 16));
        }
        float alpha[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float mn = fmaxf(m_run[j], mloc[j]);   // finite: >= 1 valid token here
          alpha[j] = exp2f(m_run[j] - mn);               // m_run = -inf -> 0
          m_run[j] = mn;
          l_run[j] *= alpha[j];
        }
#pragma unroll
        for (int mt = 0; mt < KC; ++mt) {
          o[mt][0] *= alpha[0]; o[mt][1] *= alpha[1];
          o[mt][2] *= alpha[0]; o[mt][3] *= alpha[1];
        }
        // ---- P, then O^T += V^T . P^T ----
#pragma unroll
        for (int j = 0; j < NTL; ++j) {
          if (j < my_tiles) {
            float pr[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              pr[r] = exp2f(sacc[j][r] - m_run[r & 1]);
              l_run[r & 1] += pr[r];
            }
            // S^T fragment rows are tokens, columns heads; the B operand needs
            // (k = token, n = head): transpose each 8x8 block in registers.
            const uint32_t b0 = movmatrix_trans(Mma<T>::pack(pr[0], pr[1]));
            const uint32_t b1 = movmatrix_trans(Mma<T>::pack(pr[2], pr[3]));
            const int vrow = row_lo + j * 16 + (lane & 7) + (lane >> 4) * 8;
#pragma unroll
            for (int mt = 0; mt < KC; ++mt) {
              const int d0 = mt * 16 + ((lane >> 3) & 1) * 8;
              uint32_t a[4];
              ldsm_x4_trans(vaddr + smem_off(vrow, d0), a[0], a[1], a[2], a[3]);
              Mma<T>::run(o[mt], a, b0, b1);
            }
          }
        }
      }
      __syncwarp();
      if (FUSE && patched) fence_proxy_async_smem();   // generic writes before the next TMA
      if (lane == 0) mbar_arrive(smem_u32(&empty_bar[slot]));
    }

    if (!it.last) continue;   // the segment goes on in the next piece

    // ---- segment epilogue: combine the consumer warps ----
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 4);
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 8);
      l_run[j] += __shfl_xor_sync(0xffffffffu, l_run[j], 16);
    }
    // The last consumer warp to finish the item merges all warps' partial states;
    // the others go straight on to the next item's stages, so the ring keeps
    // streaming across item boundaries.  Before overwriting its slot, a warp checks
    // (bounded wait) that the previous item has been merged; in practice that merge
    // ended a whole item earlier.
    if (item_seq > 0 && *comb_done < item_seq) {
      const unsigned long long t0 = globaltimer_ns();
      while (*comb_done < item_seq && !*abort_flag) {
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          *abort_flag = 1;
          atomicOr(p.status, kStatusWaitTimeout);
        }
      }
    }
    float* my_o = comb_o + warp * D * 8;
#pragma unroll
    for (int mt = 0; mt < KC; ++mt) {
      const int d0 = mt * 16 + g;
      my_o[d0 * 8 + 2 * c] = o[mt][0];
      my_o[d0 * 8 + 2 * c + 1] = o[mt][1];
      my_o[(d0 + 8) * 8 + 2 * c] = o[mt][2];
      my_o[(d0 + 8) * 8 + 2 * c + 1] = o[mt][3];
    }
    if (g == 0) {
      comb_m[warp * 8 + 2 * c] = m_run[0];
      comb_m[warp * 8 + 2 * c + 1] = m_run[1];
      comb_l[warp * 8 + 2 * c] = l_run[0];
      comb_l[warp * 8 + 2 * c + 1] = l_run[1];
    }
    __syncwarp();
    __threadfence_block();
    int last = 0;
    if (lane == 0) last = atomicAdd(comb_count, 1) == kConsumers - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence_block();
      const int nh = min(8, p.G - it.hg * 8);
      const bool single = it.whole;     // no other CTA or partition shares the row
      // Per-head weights once: lane n < 8 owns head n.  Warps without tokens have
      // m = -inf and weight 0.
      float wsc[kConsumers];
      float M = -INFINITY, lsum = 0.f;
      const int hn = lane & 7;
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) M = fmaxf(M, comb_m[w * 8 + hn]);
#pragma unroll
      for (int w = 0; w < kConsumers; ++w) {
        wsc[w] = exp2f(comb_m[w * 8 + hn] - M);
        lsum += comb_l[w * 8 + hn] * wsc[w];
      }
      const float inv = single ? 1.f / fmaxf(lsum, 1e-9f) : 1.f / lsum;
      // Lane = (head hn, quarter of head_dim): 8 heads x 4 lanes.
      const int dq = lane >> 3;
      const bool handoff = p.balanced && !single;
      if (handoff) {
        // Wait (bounded) until the merge warp has taken the previous segment.
        const unsigned long long t0 = globaltimer_ns();
        while (*pend_flag != 0 && !*abort_flag) {
          if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
            *abort_flag = 1;
            atomicOr(p.status, kStatusWaitTimeout);
          }
        }
        __threadfence_block();
      }
      if (handoff && hn < nh) {
        for (int d = dq; d < D; d += 4) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumers; ++w) acc += comb_o[(w * D + d) * 8 + hn] * wsc[w];
          pend_o[hn * D + d] = acc * inv;
        }
        if (dq == 0) pend_lse[hn] = M + log2f(lsum);
      } else if (hn < nh) {
        const int hq = it.kvh * p.G + it.hg * 8 + hn;
        const size_t row = (size_t)it.b * p.Hq + hq;
        // Partial index: uniform [B, Hq, max_parts]; balanced [slot][8 heads].
        const size_t pidx = p.balanced ? (size_t)it.part * 8 + hn
                                       : row * p.max_parts + it.part;
        for (int d = dq; d < D; d += 4) {
          float acc = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumers; ++w) acc += comb_o[(w * D + d) * 8 + hn] * wsc[w];
          if (single) {
            reinterpret_cast<T*>(p.out)[row * D + d] = from_f32<T>(acc * inv);
          } else {
            p.part_o[(pidx * D) + d] = acc * inv;
          }
        }
        if (!single && dq == 0) p.part_lse[pidx] = M + log2f(lsum);
      }
      if (handoff) {
        __threadfence_block();
        __syncwarp();
        if (lane == 0) *pend_flag = 1;   // the merge warp publishes it, merges when complete
      }
      __syncwarp();
      if (lane == 0) {
        *comb_count = 0;
        __threadfence_block();
        *comb_done = item_seq + 1;
      }
    }
    ++item_seq;
  }
}

}  // namespace fast

// ---------------------------------------------------------------------------
// Generic SIMT kernel: one CTA per (partition, kv head, sequence).
// ---------------------------------------------------------------------------
namespace generic {

constexpr int kChunk = 64;
constexpr int kThreads = 128;

template <typename T>
__global__ void __launch_bounds__(kThreads)
paged_decode_simt_kernel(const T* __restrict__ q, const T* __restrict__ k_pages,
                         const T* __restrict__ v_pages, const int32_t* __restrict__ block_table,
                         const int32_t* __restrict__ seq_lens, T* __restrict__ out,
                         float* __restrict__ part_o, float* __restrict__ part_lse,
                         int32_t* __restrict__ status, int Hq, int Hkv, int D, int P,
                         int max_pages, int num_pages, int Tpart, int max_parts, float scale) {
  extern __shared__ float sm[];
  const int part = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int G = Hq / Hkv;
  int L = seq_lens[b];
  if (L > max_pages * P) {
    if (threadIdx.x == 0 && part == 0 && kvh == 0) atomicOr(status, kStatusSeqLenRange);
    L = max_pages * P;
  }
  const int nparts = (L + Tpart - 1) / Tpart;
  if (part >= nparts) return;
  const int plen = part_len(L, Tpart);
  const int t0 = part * plen;
  const int t1 = min(L, t0 + plen);

  float* qs = sm;                    // [G][D]
  float* acc = qs + G * D;           // [G][D]
  float* sc = acc + G * D;           // [G][kChunk]
  float* mrun = sc + G * kChunk;     // [G]
  float* lrun = mrun + G;            // [G]
  float* alph = lrun + G;            // [G]
  __shared__ int pages[kChunk];

  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int n = idx / D, d = idx - n * D;
    qs[idx] = to_f32(q[((size_t)b * Hq + kvh * G + n) * D + d]);
    acc[idx] = 0.f;
  }
  for (int n = threadIdx.x; n < G; n += kThreads) {
    mrun[n] = -INFINITY;
    lrun[n] = 0.f;
  }
  const int32_t* bt = block_table + (size_t)b * max_pages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int c0 = t0; c0 < t1; c0 += kChunk) {
    const int nt = min(kChunk, t1 - c0);
    __syncthreads();
    for (int t = threadIdx.x; t < nt; t += kThreads) {
      int pg = bt[(c0 + t) / P];
      if (pg < 0 || pg >= num_pages) {
        atomicOr(status, kStatusBadPage);
        pg = -1;
      }
      pages[t] = pg;
    }
    __syncthreads();
    // scores s = (q . k) * scale, fp32 accumulation in head_dim order
    for (int idx = threadIdx.x; idx < G * nt; idx += kThreads) {
      const int n = idx / nt, t = idx - n * nt;
      const int pos = c0 + t;
      float s = -INFINITY;
      if (pages[t] >= 0) {
        const T* kr = k_pages + (((size_t)pages[t] * Hkv + kvh) * P + (pos % P)) * D;
        const float* qr = qs + n * D;
        float a = 0.f;
        for (int d = 0; d < D; ++d) a = fmaf(qr[d], to_f32(kr[d]), a);
        s = ref_score<T>(a, scale);
      }
      sc[n * kChunk + t] = s;
    }
    __syncthreads();
    // online softmax update per head (warp w: heads w, w+4, ...)
    for (int n = warp; n < G; n += kThreads / 32) {
      float mx = -INFINITY;
      for (int t = lane; t < nt; t += 32) mx = fmaxf(mx, sc[n * kChunk + t]);
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mold = mrun[n];
      const float mnew = fmaxf(mold, mx);
      float sum = 0.f;
      for (int t = lane; t < nt; t += 32) {
        const float e = (mnew == -INFINITY) ? 0.f : expf(sc[n * kChunk + t] - mnew);
        sc[n * kChunk + t] = e;
        sum += e;
      }
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      __syncwarp();
      if (lane == 0) {
        const float a = (mold == -INFINITY) ? 0.f : expf(mold - mnew);
        alph[n] = a;
        lrun[n] = lrun[n] * a + sum;
        mrun[n] = mnew;
      }
    }
    __syncthreads();
    // acc = acc * alpha + P . V   (threads over (head, d); V reads coalesced along d)
    for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
      const int n = idx / D, d = idx - n * D;
      float a = acc[idx] * alph[n];
      for (int t = 0; t < nt; ++t) {
        if (pages[t] < 0) continue;
        const int pos = c0 + t;
        const T* vr = v_pages + (((size_t)pages[t] * Hkv + kvh) * P + (pos % P)) * D;
        a = fmaf(sc[n * kChunk + t], to_f32(vr[d]), a);
      }
      acc[idx] = a;
    }
  }
  __syncthreads();
  const float kLog2e = 1.4426950408889634f;
  for (int idx = threadIdx.x; idx < G * D; idx += kThreads) {
    const int n = idx / D, d = idx - n * D;
    const size_t row = (size_t)b * Hq + kvh * G + n;
    if (nparts == 1) {
      out[row * D + d] = from_f32<T>(acc[idx] / fmaxf(lrun[n], 1e-9f));
    } else {
      const size_t pi = row * max_parts + part;
      part_o[pi * D + d] = acc[idx] / lrun[n];
      if (d == 0) part_lse[pi] = mrun[n] * kLog2e + log2f(lrun[n]);
    }
  }
}

size_t smem_bytes(int G, int D) {
  return sizeof(float) * (size_t)(2 * G * D + G * kChunk + 3 * G);
}

}  // namespace generic

// ---------------------------------------------------------------------------
// Log-sum-exp merge: one CTA per (b, h); threads over head_dim.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(128)
lse_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                 const int32_t* __restrict__ seq_lens, T* __restrict__ out, int Hq, int D,
                 int max_parts, int Tpart, int cap, const int32_t* __restrict__ lens_next,
                 int32_t* __restrict__ seq_lens_out) {
  pdl_wait();   // partials of the decode kernel are complete and visible
  const int h = blockIdx.x, b = blockIdx.y;
  // After a fused RoPE+append+decode the attended lengths are in lens_next; they
  // become the cache's lengths here, once the decode kernel is done reading them.
  const int L = lens_next ? lens_next[b] : min(seq_lens[b], cap);
  if (lens_next && h == 0 && threadIdx.x == 0) seq_lens_out[b] = L;
  const int n = L > 0 ? (L + Tpart - 1) / Tpart : 0;
  const size_t row = (size_t)b * Hq + h;
  if (n == 1) return;  // written directly by the decode kernel
  if (n == 0) {
    for (int d = threadIdx.x; d < D; d += blockDim.x) out[row * D + d] = from_f32<T>(0.f);
    return;
  }
  const float* lse = part_lse + row * max_parts;
  float M = -INFINITY;
  for (int i = 0; i < n; ++i) M = fmaxf(M, lse[i]);
  float wsum = 0.f;
  for (int i = 0; i < n; ++i) wsum += exp2f(lse[i] - M);
  const float inv = 1.f / wsum;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int i = 0; i < n; ++i) a = fmaf(exp2f(lse[i] - M), part_o[(row * max_parts + i) * D + d], a);
    out[row * D + d] = from_f32<T>(a * inv);
  }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// View of a page pool [num_pages * Hkv * P rows, D cols] for TMA.  D = 128: 3-D
// {64 cols, 2 halves (stride 128 B), rows (stride 256 B)}, box {64, 2, rows};
// otherwise 2-D {D cols, rows}, box {64, rows}.  128-byte swizzle either way.
static bool encode_pool_map(CUtensorMap* map, const void* base, long long nrows, int D, int rows,
                            std::string* err) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is not available from the CUDA driver";
    return false;
  }
  CUresult r;
  if (D == 128) {
    cuuint64_t dims[3] = {64u, 2u, (cuuint64_t)nrows};
    cuuint64_t strides[2] = {128u, (cuuint64_t)D * 2};
    cuuint32_t box[3] = {64u, 2u, (cuuint32_t)rows};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<void*>(base), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)nrows};
    cuuint64_t strides[1] = {(cuuint64_t)D * 2};
    cuuint32_t box[2] = {64u, (cuuint32_t)rows};
    cuuint32_t estr[2] = {1u, 1u};
    r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) {
    *err = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
    return false;
  }
  return true;
}

struct DeviceInfo {
  int sms = 0;
  int max_smem_optin = 0;
};

static DeviceInfo device_info() {
  static DeviceInfo cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev].sms == 0) {
    cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&cache[dev].max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin,
                           dev);
  }
  return cache[dev];
}


bool fast_path_applies(int dtype, int D, int P, int max_pages, int Tpart, int B,
                       const void* q, const void* kp, const void* vp) {
  if (dtype != LLMC_BF16 && dtype != LLMC_F16) return false;
  if (D != 64 && D != 128 && D != 256) return false;
  if (Tpart % fast::kStageTok) return false;
  const bool p_ok = (P == 8 || P == 16 || P == 32 || P == 64) || (P % fast::kStageTok == 0) ||
                    max_pages == 1;
  if (!p_ok) return false;
  if (B > 4096) return false;
  auto al = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  return al(q) && al(kp) && al(vp);
}

template <int D, typename T, int ST, bool FUSE>
static cudaError_t launch_fast_t(const fast::Params& p0, const void* kp, const void* vp,
                                 long long nrows, std::string* err, cudaStream_t stream) {
  fast::Params p = p0;
  const int rows = p.P >= ST ? ST : p.P;
  CUtensorMap mk, mv;
  if (!encode_pool_map(&mk, kp, nrows, D, rows, err) ||
      !encode_pool_map(&mv, vp, nrows, D, rows, err))
    return cudaErrorInvalidValue;
  const DeviceInfo di = device_info();
  constexpr int STAGE_BYTES = 2 * (D / 64) * ST * fast::kRowBytes;
  p.max_entries = (p.balanced ? p.cap_chunks * fast::kStageTok : p.T) / p.P + 2;
  const size_t fixed = 1024 /*align*/ + sizeof(float) * (fast::kConsumers * D * 8 + 16 * fast::kConsumers) +
                       2 * fast::kMaxStages * sizeof(uint64_t) +
                       sizeof(int) * (2 * p.B + 4 + 2 * p.max_entries) + 64 +
                       sizeof(int) * 32 + sizeof(float) * (8 * D + 8);   // handoff slot
  const size_t budget = (size_t)di.max_smem_optin;
  int nst = (int)((budget - fixed) / STAGE_BYTES);
  if (nst > fast::kMaxStages) nst = fast::kMaxStages;
  nst -= nst % fast::kGroups;  // each slot is owned by one consumer group
  if (nst < fast::kGroups) {
    *err = "not enough shared memory for the decode pipeline";
    return cudaErrorInvalidValue;
  }
  p.nstages = nst;
  const size_t smem = fixed + (size_t)nst * STAGE_BYTES;
  auto kern = fast::paged_decode_tma_kernel<D, T, ST, FUSE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int grid = di.sms;
  if (!p.balanced) {
    const long long upper = (long long)p.B * p.max_parts * p.Hkv * p.HG;
    if (upper < grid) grid = (int)(upper > 0 ? upper : 1);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(fast::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, mk, mv, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

static cudaError_t launch_lse_merge_ex(const float* part_o, const float* part_lse,
                                       const int32_t* seq_lens, void* out, int B, int Hq, int D,
                                       int max_parts, int Tpart, int cap, int dtype,
                                       cudaStream_t stream, const int32_t* lens_next,
                                       int32_t* seq_lens_out);

// Pieces of the balanced split are at most this many 64-token chunks (the block-table
// slice of one piece is staged in shared memory).
constexpr int kBalancedCapChunks = 32;

int balanced_grid() { return device_info().sms; }

// Work split of the fast kernel: uniform partitions of Tpart tokens, or (Tpart == 0)
// the balanced split, whose counters head the part_lse buffer.
// The balanced split keeps chunk positions in 32 bits: every row's chunks together.
static bool balanced_fits(int B, int Hkv, int HG, int max_pages, int P) {
  const long long chunks = ((long long)max_pages * P + fast::kStageTok - 1) / fast::kStageTok;
  return (long long)B * Hkv * HG * chunks < (1ll << 31) - 1;
}

static void set_split(fast::Params& p, int Tpart, float* part_o, float* part_lse) {
  p.part_o = part_o;
  if (Tpart == 0) {
    p.balanced = 1;
    p.cap_chunks = kBalancedCapChunks;
    p.counters = reinterpret_cast<int32_t*>(part_lse);
    p.part_lse = part_lse + balanced_counter_words(p.B * p.Hkv * p.HG);
    p.T = 0;
    p.max_parts = 0;
  } else {
    p.balanced = 0;
    p.cap_chunks = 0;
    p.counters = nullptr;
    p.part_lse = part_lse;
    p.T = Tpart;
    p.max_parts = (int)(((long long)p.max_pages * p.P + Tpart - 1) / Tpart);
  }
}

template <bool FUSE>
static cudaError_t launch_fast(const fast::Params& p, int dtype, int D, const void* kp,
                               const void* vp, std::string* err, cudaStream_t stream) {
  const long long nrows = (long long)p.num_pages * p.Hkv * p.P;
  if (dtype == LLMC_BF16) {
    if (D == 64) return launch_fast_t<64, __nv_bfloat16, 64, FUSE>(p, kp, vp, nrows, err, stream);
    if (D == 128) return launch_fast_t<128, __nv_bfloat16, 64, FUSE>(p, kp, vp, nrows, err, stream);
    return launch_fast_t<256, __nv_bfloat16, 32, FUSE>(p, kp, vp, nrows, err, stream);
  }
  if (D == 64) return launch_fast_t<64, __half, 64, FUSE>(p, kp, vp, nrows, err, stream);
  if (D == 128) return launch_fast_t<128, __half, 64, FUSE>(p, kp, vp, nrows, err, stream);
  return launch_fast_t<256, __half, 32, FUSE>(p, kp, vp, nrows, err, stream);
}

// Fused RoPE + page append + decode + merge (one decode launch, one merge launch).
// Returns cudaErrorNotSupported when the fast kernel does not apply to this shape;
// the caller then runs the separate kernels.
cudaError_t launch_fused_decode(const void* q_raw, const void* k_new, const void* v_new,
                                void* q_rot_out, void* kp, void* vp, const int32_t* bt,
                                int32_t* seq_lens, const void* cos_tab, const void* sin_tab,
                                int rope_max_pos, void* out, float* part_o, float* part_lse,
                                int32_t* lens_next, int32_t* status, int B, int Hq, int Hkv,
                                int D, int P, int max_pages, int num_pages, int Tpart,
                                float scale, int dtype, std::string* err, cudaStream_t stream,
                                long long q_stride, long long kv_stride, int flags) {
  if (B == 0) return cudaSuccess;
  if (!fast_path_applies(dtype, D, P, max_pages, Tpart, B, q_raw, kp, vp))
    return cudaErrorNotSupported;
  if (Tpart == 0 && !balanced_fits(B, Hkv, (Hq / Hkv + 7) / 8, max_pages, P))
    return cudaErrorNotSupported;
  const int G = Hq / Hkv;
  fast::Params p;
  p.q = q_raw; p.out = out; p.block_table = bt;
  p.q_stride = q_stride; p.kv_stride = kv_stride;
  p.seq_lens = seq_lens; p.status = status;
  p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = G; p.HG = (G + 7) / 8; p.P = P;
  p.max_pages = max_pages; p.num_pages = num_pages;
  set_split(p, Tpart, part_o, part_lse);
  p.nstages = 0; p.scale_log2 = scale * 1.4426950408889634f; p.scale = scale;
  p.k_new = k_new; p.v_new = v_new; p.cos_tab = cos_tab; p.sin_tab = sin_tab;
  p.k_pages = kp; p.v_pages = vp; p.q_rot_out = q_rot_out; p.lens_next = lens_next;
  p.rope_max_pos = rope_max_pos;
  p.seq_lens_out = seq_lens;
  p.early = (flags & LLMC_DECODE_EARLY_TABLES) && p.balanced ? 1 : 0;
  cudaError_t e = launch_fast<true>(p, dtype, D, kp, vp, err, stream);
  if (e != cudaSuccess) return e;
  if (p.balanced) return cudaSuccess;   // merged and published inside the decode kernel
  return launch_lse_merge_ex(part_o, part_lse, seq_lens, out, B, Hq, D, p.max_parts, Tpart,
                             p.max_parts * Tpart, dtype, stream, lens_next, seq_lens);
}

cudaError_t launch_paged_decode(const void* q, const void* kp, const void* vp, const int32_t* bt,
                                const int32_t* seq_lens, void* out, float* part_o,
                                float* part_lse, int32_t* status, int B, int Hq, int Hkv, int D,
                                int P, int max_pages, int num_pages, int Tpart, float scale,
                                int dtype, int flags, std::string* err, cudaStream_t stream) {
  const int G = Hq / Hkv;
  if (B == 0) return cudaSuccess;
  const bool fast_ok = !(flags & LLMC_DECODE_FORCE_GENERIC) &&
                       fast_path_applies(dtype, D, P, max_pages, Tpart, B, q, kp, vp) &&
                       (Tpart > 0 || balanced_fits(B, Hkv, (G + 7) / 8, max_pages, P));
  if (Tpart == 0 && !fast_ok) {
    *err = "the balanced split (partition_tokens 0) needs the TMA kernel's shapes";
    return cudaErrorNotSupported;
  }
  const int max_parts = Tpart > 0 ? (int)(((long long)max_pages * P + Tpart - 1) / Tpart) : 0;
  if (fast_ok) {
    fast::Params p;
    p.q = q; p.out = out; p.block_table = bt;
    p.q_stride = (long long)Hq * D; p.kv_stride = 0;
    p.seq_lens = seq_lens; p.status = status;
    p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = G; p.HG = (G + 7) / 8; p.P = P;
    p.max_pages = max_pages; p.num_pages = num_pages;
    set_split(p, Tpart, part_o, part_lse);
    p.nstages = 0; p.scale_log2 = scale * 1.4426950408889634f; p.scale = scale;
    p.k_new = p.v_new = p.cos_tab = p.sin_tab = nullptr;
    p.k_pages = p.v_pages = p.q_rot_out = nullptr;
    p.lens_next = nullptr;
    p.rope_max_pos = 0;
    p.seq_lens_out = nullptr;
    p.early = (flags & LLMC_DECODE_EARLY_TABLES) && p.balanced ? 1 : 0;
    return launch_fast<false>(p, dtype, D, kp, vp, err, stream);
  }
  // generic SIMT path
  const size_t smem = generic::smem_bytes(G, D);
  dim3 grid(max_parts, Hkv, B);
  if (max_parts > 65535 * 1024 || Hkv > 65535 || B > 65535) {
    *err = "grid too large for the generic decode kernel";
    return cudaErrorInvalidValue;
  }
#define LLMC_GEN(TT)                                                                          \
  do {                                                                                        \
    auto k = generic::paged_decode_simt_kernel<TT>;                                           \
    if (smem > 48 * 1024) {                                                                   \
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                           (int)smem);                                        \
      if (e != cudaSuccess) return e;                                                         \
    }                                                                                         \
    k<<<grid, generic::kThreads, smem, stream>>>((const TT*)q, (const TT*)kp, (const TT*)vp,  \
                                                 bt, seq_lens, (TT*)out, part_o, part_lse,    \
                                                 status, Hq, Hkv, D, P, max_pages, num_pages, \
                                                 Tpart, max_parts, scale);                    \
  } while (0)
  if (dtype == LLMC_F32) LLMC_GEN(float);
  else if (dtype == LLMC_F16) LLMC_GEN(__half);
  else LLMC_GEN(__nv_bfloat16);
#undef LLMC_GEN
  return cudaGetLastError();
}

static cudaError_t launch_lse_merge_ex(const float* part_o, const float* part_lse,
                                       const int32_t* seq_lens, void* out, int B, int Hq, int D,
                                       int max_parts, int Tpart, int cap, int dtype,
                                       cudaStream_t stream, const int32_t* lens_next,
                                       int32_t* seq_lens_out);

cudaError_t launch_lse_merge(const float* part_o, const float* part_lse, const int32_t* seq_lens,
                             void* out, int B, int Hq, int D, int max_parts, int Tpart, int cap,
                             int dtype, cudaStream_t stream) {
  if (Tpart == 0) return cudaSuccess;   // the balanced decode kernel merges its own rows
  return launch_lse_merge_ex(part_o, part_lse, seq_lens, out, B, Hq, D, max_parts, Tpart, cap,
                             dtype, stream, nullptr, nullptr);
}

static cudaError_t launch_lse_merge_ex(const float* part_o, const float* part_lse,
                                       const int32_t* seq_lens, void* out, int B, int Hq, int D,
                                       int max_parts, int Tpart, int cap, int dtype,
                                       cudaStream_t stream, const int32_t* lens_next,
                                       int32_t* seq_lens_out) {
  if (B == 0 || Hq == 0) return cudaSuccess;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(Hq, B);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  if (dtype == LLMC_F32)
    e = cudaLaunchKernelEx(&cfg, lse_merge_kernel<float>, part_o, part_lse, seq_lens,
                           (float*)out, Hq, D, max_parts, Tpart, cap, lens_next, seq_lens_out);
  else if (dtype == LLMC_F16)
    e = cudaLaunchKernelEx(&cfg, lse_merge_kernel<__half>, part_o, part_lse, seq_lens,
                           (__half*)out, Hq, D, max_parts, Tpart, cap, lens_next, seq_lens_out);
  else
    e = cudaLaunchKernelEx(&cfg, lse_merge_kernel<__nv_bfloat16>, part_o, part_lse, seq_lens,
                           (__nv_bfloat16*)out, Hq, D, max_parts, Tpart, cap, lens_next,
                           seq_lens_out);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace llmc
