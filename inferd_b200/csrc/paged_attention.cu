// paged_attention.cu -- paged GQA attention over the block-table KV pool.
//
// Fast path (bf16/f16, head_dim 128, block_size 16, q_len * group <= 32):
//   A persistent kernel of independent warps.  The (sequence, kv-head) page lists are
//   laid end to end into one page axis of T = num_kv_heads * sum_b ceil(L_b / 16) pages,
//   and warp w of the U warps in the grid streams pages [w*T/U, (w+1)*T/U), so every warp
//   moves the same number of bytes however uneven the context lengths are.
//
//   Each warp feeds itself: it reads 32 block ids at a time with one coalesced load
//   (prefetching the next 32), lane 0 issues TMA 2-D tiled loads (128-byte swizzle,
//   evict-first L2 policy) of 4 KiB K and V pages into the warp's own 3-stage shared-
//   memory ring, and the warp computes S = K Q^T and O^T += V^T P^T on mma.sync m16n8k16
//   with fp32 accumulators, an online softmax in base 2 with warp-shuffle column maxima,
//   and movmatrix to turn the P accumulator into an MMA operand.  All query rows that
//   share a kv head (group heads x q_len queries) ride in the MMA's N dimension, so each
//   K/V byte is read from HBM once.  Warps never wait for one another: there is no
//   block-level barrier after set-up.
//
//   A (sequence, kv head) segment that lies inside one warp's range is normalised and
//   stored directly.  A segment cut by warp ranges gets one partial (m, l, O) per warp.
//   With one n-tile (decode) the warp that finishes the segment last (atomic ticket, no
//   spinning) merges them; with several (verify windows) merge_cut_segments_kernel, launched
//   right after, merges every cut segment in parallel.
//
// Generic path (fp32 and any other size): one CTA per (sequence, query row), fp32 CUDA
// core arithmetic.  Used for fp32 pools and small head dims such as the reference's
// own unit tests; it is not tuned.
//
// Numerics follow core/paged_attn.py:64-106 (GQA through repeat_interleave order,
// default scale 1/sqrt(head_dim), fp32 softmax, probabilities rounded to the working
// dtype before P.V) except that Q.K is accumulated in fp32 rather than rounded to the
// working dtype.
#include <atomic>
#include <type_traits>

#include <mutex>

#include "common.cuh"
#include "runtime.cuh"

namespace inferd {
namespace {

constexpr int kHeadDim = 128;
constexpr int kPage = 16;                    // tokens per KV block
constexpr int kHalfBytes = 2048;             // one TMA box: 16 rows x 64 elements x 2 B
constexpr int kStageBytes = 4 * kHalfBytes;  // K lo/hi, V lo/hi halves of one page
constexpr int kWarps = 4;                    // warps per CTA
constexpr int kCtasPerSm = 2;
constexpr int kMaxSeqsFast = 1024;  // sequences per launch (larger batches are chunked)
constexpr int kMaxKvHeadsFast = 128;
constexpr int kMaxRowsFast = 32;    // q_len * group rows per (sequence, kv head)
constexpr float kLog2e = 1.4426950408889634f;

#ifndef INFERD_STAGES_PER_WARP
#define INFERD_STAGES_PER_WARP 3  // pages in flight per warp (3 x 8 KiB)
#endif
constexpr int kStagesPerWarp = INFERD_STAGES_PER_WARP;

// query rows per (sequence, kv head), rounded up to whole 8-column MMA tiles
__host__ __device__ constexpr int nq_pad(int nq) { return ((nq + 7) / 8) * 8; }

struct FastParams {
  void* out;
  const void* query;
  const void* block_tables;
  int64_t bt_stride;
  int32_t bt_bytes;
  const int32_t* context_lens;
  int32_t max_context_len;
  int32_t num_seqs, q_len, num_q_heads, num_kv_heads, group, nq;
  int64_t num_blocks;
  float scale_log2;
  int32_t* counters;  // per (sequence, kv head) ticket counters / cut markers, 0 between launches
  float* part_ml;     // [slot][NQP][2]    (m, l) per query row
  float* part_o;      // [slot][128][NQP]  unnormalised O, query row fastest
  int32_t* error_word;
  // Output gather fused into the epilogue: once a (sequence, kv head) segment's output rows
  // are in out, they are copied to peer_out[i] + peer_offset + (their index in out) for
  // i < num_peers -- each rank's gather slot, through NVLink for peers -- as 16-byte
  // vectors.  num_peers == 0: out only.
  void* const* peer_out;
  int32_t num_peers;
  int64_t peer_offset;
};

// Copy the output rows of segment (b, h) -- q_len runs of group * 128 contiguous elements --
// from out to every gather destination; thread t of nthreads.  The caller makes the rows'
// stores visible to these threads first (__syncwarp / __syncthreads).
template <typename T>
__device__ __forceinline__ void copy_segment_to_peers(const FastParams& p, const T* optr, int b,
                                                      int h, int t, int nthreads) {
  constexpr int kVec = 16 / sizeof(T);
  const int per = p.group * (kHeadDim / kVec);  // vectors per query position
  for (int i = t; i < per * p.q_len; i += nthreads) {
    const int qi = i / per, k = i - qi * per;
    const int64_t base =
        ((static_cast<int64_t>(b) * p.q_len + qi) * p.num_q_heads + static_cast<int64_t>(h) * p.group) * kHeadDim;
    const uint4 v = reinterpret_cast<const uint4*>(optr + base)[k];
    for (int r = 0; r < p.num_peers; ++r)
      reinterpret_cast<uint4*>(static_cast<T*>(p.peer_out[r]) + p.peer_offset + base)[k] = v;
  }
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// Context length of sequence b, clamped to what its block-table row can address.
__device__ __forceinline__ int seq_len_of(const FastParams& p, int b, bool report) {
  int L = p.context_lens != nullptr ? __ldg(p.context_lens + b) : p.max_context_len;
  if (L < 0) L = 0;
  const int64_t cap = p.bt_stride * kPage;
  if (L > cap) {
    if (report) report_error(p.error_word, INFERD_ERR_DEVICE_INDEX);
    L = static_cast<int>(cap);
  }
  return L;
}

__device__ __forceinline__ int64_t block_id(const FastParams& p, int b, int page) {
  const int64_t i = static_cast<int64_t>(b) * p.bt_stride + page;
  return p.bt_bytes == 8 ? __ldg(static_cast<const int64_t*>(p.block_tables) + i)
                         : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(p.block_tables) + i));
}

// Largest b in [0, B) with prefix[b] <= q.
__device__ __forceinline__ int find_seq(const int* prefix, int B, int64_t q) {
  int lo = 0, hi = B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= q) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Unit (warp) whose balanced range [u*T/U, (u+1)*T/U) contains global page g.
__device__ __forceinline__ int unit_of(int64_t g, int64_t T, int U) {
  int64_t u = ((g + 1) * U + T - 1) / T - 1;
  if (u < 0) u = 0;
  if (u > U - 1) u = U - 1;
  return static_cast<int>(u);
}

// Pages per sequence and their exclusive prefix over the launch's sequences, by a block
// scan over NTHREADS threads: prefix[b] = pages of sequences [0, b), prefix[B] = total.
// Ends with a block barrier.
template <int NTHREADS>
__device__ __forceinline__ void page_prefix(const FastParams& p, int* prefix, int* warp_tot) {
  constexpr int kW = NTHREADS / 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = p.num_seqs;
  const int chunk = (B + NTHREADS - 1) / NTHREADS;
  const int b0 = min(B, tid * chunk), b1 = min(B, b0 + chunk);
  int local = 0;
  for (int b = b0; b < b1; ++b) local += (seq_len_of(p, b, true) + kPage - 1) / kPage;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int run = incl - local;
  int total = 0;
  for (int w = 0; w < kW; ++w) {
    if (w < warp) run += warp_tot[w];
    total += warp_tot[w];
  }
  for (int b = b0; b < b1; ++b) {
    prefix[b] = run;
    run += (seq_len_of(p, b, false) + kPage - 1) / kPage;
  }
  if (tid == 0) prefix[B] = total;
  __syncthreads();
}

// Query-row fragments (MMA B operand, d x rows) of one segment, read from global memory:
// b0 = rows n = nt*8 + lane/4, d = kk*16 + 2*(lane%4) + {0,1}; b1 = the same at d + 8.
template <typename T, int NT>
__device__ __forceinline__ void load_q_frags(uint32_t (&qf)[8][NT][2], const T* qptr,
                                             const FastParams& p, int b, int h, int lane) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int c = nt * 8 + (lane >> 2);
    const bool live = c < p.nq;
    const int qi = live ? c / p.group : 0, gi = live ? c - qi * p.group : 0;
    const uint32_t* row = reinterpret_cast<const uint32_t*>(
        qptr + ((static_cast<int64_t>(b) * p.q_len + qi) * p.num_q_heads + h * p.group + gi) * kHeadDim);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qf[kk][nt][0] = live ? __ldg(row + kk * 8 + (lane & 3)) : 0u;
      qf[kk][nt][1] = live ? __ldg(row + kk * 8 + 4 + (lane & 3)) : 0u;
    }
  }
}

template <bool kBf16, int NT, int STAGES>
__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
    paged_attn_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap, const FastParams p) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  constexpr int NQP = NT * 8;
  constexpr int kThreads = kWarps * 32;

  extern __shared__ uint8_t smem_raw[];
  __shared__ int warp_tot[kWarps];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars_all = reinterpret_cast<uint64_t*>(smem + kWarps * STAGES * kStageBytes);
  int* prefix = reinterpret_cast<int*>(bars_all + kWarps * STAGES);  // [B + 1]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int B = p.num_seqs, Hkv = p.num_kv_heads;

  page_prefix<kThreads>(p, prefix, warp_tot);
  // No block-level synchronisation below this point: every warp runs on its own.

  const int64_t T_pages = static_cast<int64_t>(Hkv) * prefix[B];
  const int U = static_cast<int>(min64(static_cast<int64_t>(gridDim.x) * kWarps, max64(T_pages, 1)));
  const int w = blockIdx.x * kWarps + warp;
  if (w >= U) return;

  // Sequences without keys: softmax over an empty set -> zero output rows.
  for (int b = w; b < B; b += U) {
    if (prefix[b + 1] != prefix[b]) continue;
    const int64_t n16 = static_cast<int64_t>(p.q_len) * p.num_q_heads * kHeadDim / 8;
    uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(p.out) +
                                          static_cast<int64_t>(b) * p.q_len * p.num_q_heads * kHeadDim);
    for (int64_t i = lane; i < n16; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    for (int i = 0; i < p.num_peers; ++i) {
      uint4* pd = reinterpret_cast<uint4*>(static_cast<T*>(p.peer_out[i]) + p.peer_offset +
                                           static_cast<int64_t>(b) * p.q_len * p.num_q_heads * kHeadDim);
      for (int64_t j = lane; j < n16; j += 32) pd[j] = make_uint4(0, 0, 0, 0);
    }
  }
  if (T_pages == 0) return;

  const int64_t g0 = static_cast<int64_t>(w) * T_pages / U;
  const int64_t g1 = static_cast<int64_t>(w + 1) * T_pages / U;
  const int n_pages = static_cast<int>(g1 - g0);
  uint8_t* stages = smem + warp * STAGES * kStageBytes;
  uint64_t* full = bars_all + warp * STAGES;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  __syncwarp();

  const uint64_t policy = l2_policy_evict_first();
  const T* qptr = static_cast<const T*>(p.query);
  T* optr = static_cast<T*>(p.out);
  const int mrow = lane & 7, msel = lane >> 3;

  // pool row (block * Hkv + head) * 16 of global page g
  auto row_of = [&](int64_t g) -> int32_t {
    const int b = find_seq(prefix, B, g / Hkv);
    const int pb = prefix[b + 1] - prefix[b];
    const int64_t off = g - static_cast<int64_t>(Hkv) * prefix[b];
    const int h = static_cast<int>(off / pb);
    const int page = static_cast<int>(off - static_cast<int64_t>(h) * pb);
    int64_t blk = block_id(p, b, page);
    if (blk < 0 || blk >= p.num_blocks) {
      report_error(p.error_word, INFERD_ERR_DEVICE_INDEX);
      blk = 0;
    }
    return static_cast<int32_t>((blk * Hkv + h) * kPage);
  };
  // Block ids of this warp's pages, 32 per register batch: rows_cur holds pages
  // [32k, 32k+32) of the warp's range, rows_next the following 32.
  int32_t rows_cur = lane < n_pages ? row_of(g0 + lane) : 0;
  int32_t rows_next = 32 + lane < n_pages ? row_of(g0 + 32 + lane) : 0;
  bool abort = false;

  // Issue local page j (all lanes call; rows looked up by shuffle; lane 0 issues).
  auto issue_page = [&](int j, int cur_batch) {
    const int32_t rc = __shfl_sync(0xffffffffu, rows_cur, j & 31);
    const int32_t rn = __shfl_sync(0xffffffffu, rows_next, j & 31);
    const int32_t r = (j >> 5) == cur_batch ? rc : rn;
    if (lane == 0) {
      const int s = j % STAGES;
      uint8_t* st = stages + s * kStageBytes;
      mbar_arrive_expect_tx(&full[s], kStageBytes);
      tma_load_2d(st, &kmap, 0, r, &full[s], policy);
      tma_load_2d(st + kHalfBytes, &kmap, 64, r, &full[s], policy);
      tma_load_2d(st + 2 * kHalfBytes, &vmap, 0, r, &full[s], policy);
      tma_load_2d(st + 3 * kHalfBytes, &vmap, 64, r, &full[s], policy);
    }
  };
  int issued = 0;
  for (; issued < STAGES && issued < n_pages; ++issued) issue_page(issued, 0);

  // ---- current segment (sequence b, kv head h) and its state
  int b = find_seq(prefix, B, g0 / Hkv);
  int pb = prefix[b + 1] - prefix[b];
  int64_t seg_start = static_cast<int64_t>(Hkv) * prefix[b];
  int h = static_cast<int>((g0 - seg_start) / pb);
  seg_start += static_cast<int64_t>(h) * pb;
  int64_t seg_end = seg_start + pb;
  int L = seq_len_of(p, b, false);
  int64_t piece_start = g0;

  uint32_t qf[8][NT][2];
  int lim[NT][2];
  float m[NT][2], l[NT][2], o[8][NT][4];

  auto begin_segment = [&]() {
    load_q_frags<T, NT>(qf, qptr, p, b, h, lane);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = nt * 8 + 2 * (lane & 3) + j;
        lim[nt][j] = c < p.nq ? L - p.q_len + c / p.group : -1;
        m[nt][j] = -INFINITY;
        l[nt][j] = 0.f;
      }
#pragma unroll
      for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[mt][nt][e] = 0.f;
    }
  };

  // Segments this warp merges after its page loop: at most the one its range opens
  // inside and the one it closes inside.
  int n_merge = 0, merge_b0 = 0, merge_h0 = 0, merge_b1 = 0, merge_h1 = 0;

  // Finish the piece [piece_start, piece_end) of the current segment: store the output
  // if the piece is the whole segment, else publish a partial and take a ticket.
  auto end_piece = [&](int64_t piece_end) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float v = l[nt][j];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        l[nt][j] = v;
      }
    const int seg_id = b * Hkv + h;
    if (piece_start == seg_start && piece_end == seg_end) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = nt * 8 + 2 * (lane & 3) + (e & 1);
          if (c >= p.nq) continue;
          const float lv = l[nt][e & 1];
          const float inv = lv > 0.f ? 1.f / lv : 0.f;
          const int qi = c / p.group, gi = c - qi * p.group;
          const int64_t row = ((static_cast<int64_t>(b) * p.q_len + qi) * p.num_q_heads + h * p.group + gi) * kHeadDim;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt)
            optr[row + mt * 16 + (lane >> 2) + ((e >> 1) << 3)] = from_f32<T>(o[mt][nt][e] * inv);
        }
      if (p.num_peers > 0) {
        __syncwarp();
        copy_segment_to_peers<T>(p, optr, b, h, lane, 32);
      }
      return;
    }
    // partial: slot = unit + segment id is unique (units and segments are both monotone
    // along the page axis), at most U + segments slots
    const int64_t slot = static_cast<int64_t>(w) + seg_id;
    float* po = p.part_o + slot * kHeadDim * NQP;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < 8; ++mt)
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int d = mt * 16 + (lane >> 2) + hi * 8;
          *reinterpret_cast<float2*>(po + d * NQP + nt * 8 + 2 * (lane & 3)) =
              make_float2(o[mt][nt][2 * hi], o[mt][nt][2 * hi + 1]);
        }
    if (lane < 4) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int c = nt * 8 + 2 * lane + j;
          *reinterpret_cast<float2*>(p.part_ml + (slot * NQP + c) * 2) = make_float2(m[nt][j], l[nt][j]);
        }
    }
    const int u_first = unit_of(seg_start, T_pages, U);
    const int u_last = unit_of(seg_end - 1, T_pages, U);
    if constexpr (NT > 1) {
      // partials only: merge_cut_segments_kernel merges every cut segment after this grid.
      // Every piece of the segment stores the same marker (piece count, first unit); both
      // fit (the host keeps the grid below 2048 warps).
      if (lane == 0) p.counters[seg_id] = ((u_last - u_first + 1) << 20) | u_first;
      return;
    }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(p.counters + seg_id, 1) == u_last - u_first;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    // this warp finished the segment last: merge it after the page loop
    if (n_merge == 0) { merge_b0 = b; merge_h0 = h; } else { merge_b1 = b; merge_h1 = h; }
    ++n_merge;
  };

  // ---- merge the partials of segment (mb, mh).  Merges run after the warp's page loop,
  // where none of the loop's registers are live; those of the segments cut at the end of
  // warp ranges run after every warp's loop, so each dependent L2 round trip here
  // lengthens the launch: a piece's (m, l) is read once, and two pieces' O partials are
  // in flight together.
  auto merge_segment = [&](int mb, int mh) {
    __threadfence();
    const int mpb = prefix[mb + 1] - prefix[mb];
    const int64_t mstart = static_cast<int64_t>(Hkv) * prefix[mb] + static_cast<int64_t>(mh) * mpb;
    const int u_first = unit_of(mstart, T_pages, U);
    const int u_last = unit_of(mstart + mpb - 1, T_pages, U);
    const int seg_id = mb * Hkv + mh;
    const int np = u_last - u_first + 1;
    const int cp = 2 * (lane & 3);
    for (int nt = 0; nt < NT; ++nt) {
      // column maxima over all pieces, 8 columns of this n-tile; lane q keeps piece q's
      // (m, l) of the first 32 pieces in mq / lq
      float M[8], Ls[8], mq[8], lq[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) M[c] = -INFINITY, Ls[c] = 0.f, mq[c] = -INFINITY, lq[c] = 0.f;
      for (int p0 = 0; p0 < np; p0 += 32) {
        if (p0 + lane < np) {
          const float2* ml = reinterpret_cast<const float2*>(
              p.part_ml + ((static_cast<int64_t>(u_first) + p0 + lane + seg_id) * NQP + nt * 8) * 2);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float2 v = __ldcg(ml + c);
            M[c] = fmaxf(M[c], v.x);
            if (p0 == 0) { mq[c] = v.x; lq[c] = v.y; }
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) M[c] = fmaxf(M[c], __shfl_xor_sync(0xffffffffu, M[c], o2));
      // each lane: the two columns cp, cp + 1 of this n-tile and rows d = k*8 + lane/4
      float2 acc[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) acc[k] = make_float2(0.f, 0.f);
      for (int p0 = 0; p0 < np; p0 += 32) {
        const bool have = p0 + lane < np;
        if (p0 > 0) {
          const float2* ml = reinterpret_cast<const float2*>(
              p.part_ml + ((static_cast<int64_t>(u_first) + p0 + lane + seg_id) * NQP + nt * 8) * 2);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float2 v = have ? __ldcg(ml + c) : make_float2(-INFINITY, 0.f);
            mq[c] = v.x;
            lq[c] = v.y;
          }
        }
        // lane q of the chunk holds piece p0+q's weights exp2(m - M) for all 8 columns
        float fq[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          fq[c] = ex2(mq[c] - (M[c] == -INFINITY ? 0.f : M[c]));
          Ls[c] += lq[c] * fq[c];
        }
        const int nq_chunk = min(32, np - p0);
        for (int q0 = 0; q0 < nq_chunk; q0 += 2) {
          float2 v[2][16];
          float f0[2], f1[2];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int q = q0 + i;
            f0[i] = f1[i] = 0.f;
#pragma unroll
            for (int c = 0; c < 8; c += 2) {
              const float a0 = __shfl_sync(0xffffffffu, fq[c], q & 31);
              const float a1 = __shfl_sync(0xffffffffu, fq[c + 1], q & 31);
              if (c == cp) { f0[i] = a0; f1[i] = a1; }
            }
            if (q < nq_chunk) {
              const float* po2 = p.part_o + (static_cast<int64_t>(u_first) + p0 + q + seg_id) * kHeadDim * NQP + nt * 8 + cp;
#pragma unroll
              for (int k = 0; k < 16; ++k)
                v[i][k] = __ldcg(reinterpret_cast<const float2*>(po2 + (k * 8 + (lane >> 2)) * NQP));
            }
          }
          // pieces in order, as one piece at a time would add them
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (q0 + i < nq_chunk) {
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                acc[k].x += f0[i] * v[i][k].x;
                acc[k].y += f1[i] * v[i][k].y;
              }
            }
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) Ls[c] += __shfl_xor_sync(0xffffffffu, Ls[c], o2);
      float L0 = 0.f, L1 = 0.f;
#pragma unroll
      for (int c = 0; c < 8; c += 2)
        if (c == cp) { L0 = Ls[c]; L1 = Ls[c + 1]; }
      const float i0 = L0 > 0.f ? 1.f / L0 : 0.f, i1 = L1 > 0.f ? 1.f / L1 : 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = nt * 8 + cp + j;
        if (c >= p.nq) continue;
        const int qi = c / p.group, gi = c - qi * p.group;
        const int64_t row = ((static_cast<int64_t>(mb) * p.q_len + qi) * p.num_q_heads + mh * p.group + gi) * kHeadDim;
#pragma unroll
        for (int k = 0; k < 16; ++k)
          optr[row + k * 8 + (lane >> 2)] = from_f32<T>(j == 0 ? acc[k].x * i0 : acc[k].y * i1);
      }
    }
    if (p.num_peers > 0) {
      __syncwarp();
      copy_segment_to_peers<T>(p, optr, mb, mh, lane, 32);
    }
    if (lane == 0) p.counters[seg_id] = 0;
  };

  begin_segment();
  int cur_batch = 0;
  for (int j = 0; j < n_pages; ++j) {
    const int64_t g = g0 + j;
    if (g == seg_end) {
      // next segment: close this piece, advance (sequence, head)
      end_piece(g);
      ++h;
      if (h == Hkv) {
        h = 0;
        do { ++b; } while (prefix[b + 1] == prefix[b]);
        L = seq_len_of(p, b, false);
      }
      pb = prefix[b + 1] - prefix[b];
      seg_start = g;
      seg_end = g + pb;
      piece_start = g;
      begin_segment();
    }
    if ((j >> 5) != cur_batch) {  // rotate the block-id batches
      cur_batch = j >> 5;
      rows_cur = rows_next;
      const int nxt = (cur_batch + 1) * 32 + lane;
      rows_next = nxt < n_pages ? row_of(g0 + nxt) : 0;
    }
    const int s = j % STAGES;
    bool ok = !abort;
    if (ok && !mbar_wait(&full[s], (j / STAGES) & 1u)) ok = false;
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (!ok) {
      if (!abort && lane == 0) report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
      abort = true;
    } else {
      const uint32_t kbase = smem_u32(stages + s * kStageBytes);
      const uint32_t vbase = kbase + 2 * kHalfBytes;
      const int tok0 = static_cast<int>(g - seg_start) * kPage;

      // S[token][col] = K Q^T (fp32); even and odd k-steps in separate accumulators
      float sa[NT][4], sb[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int tok = ((msel & 1) << 3) + mrow;
        const int ch = ((kk & 3) << 1) + (msel >> 1);
        uint32_t a[4];
        ldmatrix_x4(a, kbase + (kk >> 2) * kHalfBytes + tok * 128 + ((ch ^ (tok & 7)) << 4));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (kk & 1) mma_16816<kBf16>(sb[nt], a, qf[kk][nt][0], qf[kk][nt][1]);
          else mma_16816<kBf16>(sa[nt], a, qf[kk][nt][0], qf[kk][nt][1]);
        }
      }

      // scale to base 2, causal / length mask
      const bool need_mask = tok0 + kPage - 1 > L - p.q_len;
      const int t_lo = tok0 + (lane >> 2);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float v = (sa[nt][e] + sb[nt][e]) * p.scale_log2;
          if (need_mask) {
            const int t = t_lo + ((e >> 1) << 3);
            if (t > lim[nt][e & 1]) v = -INFINITY;
          }
          sa[nt][e] = v;
        }

      // online softmax: column max over the 16 tokens (lanes sharing lane & 3)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          float mx = fmaxf(sa[nt][jj], sa[nt][jj + 2]);
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
          const float mnew = fmaxf(m[nt][jj], mx);
          const float mref = mnew == -INFINITY ? 0.f : mnew;
          const float alpha = ex2(m[nt][jj] - mref);
          m[nt][jj] = mnew;
          const float p0 = ex2(sa[nt][jj] - mref), p1 = ex2(sa[nt][jj + 2] - mref);
          sa[nt][jj] = p0;
          sa[nt][jj + 2] = p1;
          l[nt][jj] = l[nt][jj] * alpha + p0 + p1;
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[mt][nt][jj] *= alpha;
            o[mt][nt][jj + 2] *= alpha;
          }
        }

      // P^T fragments (tokens x cols) in the working dtype
      uint32_t pf[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        pf[nt][0] = movmatrix_trans(pack2<kBf16>(sa[nt][0], sa[nt][1]));
        pf[nt][1] = movmatrix_trans(pack2<kBf16>(sa[nt][2], sa[nt][3]));
      }

      // O^T[d][col] += V^T P^T ; rows of V past the sequence end hold stale pool bytes
      const bool vmask = tok0 + kPage > L;
      const int ta = tok0 + 2 * (lane & 3);
      const uint32_t m01 = (ta < L ? 0x0000ffffu : 0u) | (ta + 1 < L ? 0xffff0000u : 0u);
      const uint32_t m23 = (ta + 8 < L ? 0x0000ffffu : 0u) | (ta + 9 < L ? 0xffff0000u : 0u);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        const int tok = ((msel >> 1) << 3) + mrow;
        const int ch = ((mt & 3) << 1) + (msel & 1);
        uint32_t a[4];
        ldmatrix_x4_trans(a, vbase + (mt >> 2) * kHalfBytes + tok * 128 + ((ch ^ (tok & 7)) << 4));
        if (vmask) {
          a[0] &= m01;
          a[1] &= m01;
          a[2] &= m23;
          a[3] &= m23;
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_16816<kBf16>(o[mt][nt], a, pf[nt][0], pf[nt][1]);
      }
    }
    // refill the stage just consumed with page j + STAGES (the warp's reads of it are
    // complete: every ldmatrix result has been consumed by an MMA above)
    __syncwarp();
    if (!abort && issued < n_pages) {
      issue_page(issued, cur_batch);
      ++issued;
    }
  }
  // (also after an abort, so the ticket counters return to zero)
  end_piece(g1);
  if constexpr (NT == 1) {
    if (n_merge > 0) merge_segment(merge_b0, merge_h0);
    if (n_merge > 1) merge_segment(merge_b1, merge_h1);
  }
  // the merge kernel that follows (deferred merging) may be scheduled once every CTA has a
  // warp past this point; it waits for the whole grid before it reads anything
  grid_launch_dependents();

  // Drain: never leave the warp with a TMA write still in flight into its smem.
  if (abort && lane == 0) {
    for (int s = 0; s < STAGES && s < issued; ++s) {
      const int rounds = (issued - s + STAGES - 1) / STAGES;
      mbar_wait(&full[s], static_cast<uint32_t>((rounds - 1) & 1));
    }
  }
}

// One CTA per (sequence, kv head) segment; the segments the attention grid cut into pieces
// (marker in counters) are merged, the others skipped.  Thread d owns row d of O for all
// NQP query rows.  Launched after paged_attn_tc_kernel when the pieces carry several
// n-tiles: there one warp merging a segment alone at the end of the attention grid took
// 6-12 us of dependent L2 round trips, while here every segment merges at once.
template <typename T, int NQP>
__global__ void __launch_bounds__(kHeadDim) merge_cut_segments_kernel(const FastParams p) {
  grid_dependency_wait();  // the attention grid's partials and markers
  const int seg_id = blockIdx.x;
  const int code = p.counters[seg_id];
  if (code == 0) return;
  const int u_first = code & 0xfffff, np = code >> 20;
  const int b = seg_id / p.num_kv_heads, h = seg_id - b * p.num_kv_heads;
  const int d = threadIdx.x;
  __shared__ float2 mls[32][NQP];  // (m, l) of up to 32 pieces, loaded in one round trip
  __shared__ float f[32][NQP];     // their weights exp2(m - M)
  __shared__ float Ms[NQP], Linv[NQP];
  // slots of the pieces: unit + segment id, consecutive units
  const float2* ml = reinterpret_cast<const float2*>(p.part_ml) + (static_cast<int64_t>(u_first) + seg_id) * NQP;
  const float* po = p.part_o + (static_cast<int64_t>(u_first) + seg_id) * kHeadDim * NQP;
  auto load_ml = [&](int q0, int nqc) {
    for (int i = d; i < nqc * NQP; i += kHeadDim) mls[i / NQP][i % NQP] = __ldcg(ml + q0 * NQP + i);
  };
  // column maxima over all pieces
  float mx = -INFINITY;
  for (int q0 = 0; q0 < np; q0 += 32) {
    const int nqc = min(32, np - q0);
    __syncthreads();
    load_ml(q0, nqc);
    __syncthreads();
    if (d < NQP)
      for (int q = 0; q < nqc; ++q) mx = fmaxf(mx, mls[q][d].x);
  }
  if (d < NQP) Ms[d] = mx == -INFINITY ? 0.f : mx;
  float L = 0.f, acc[NQP];
#pragma unroll
  for (int c = 0; c < NQP; ++c) acc[c] = 0.f;
  for (int q0 = 0; q0 < np; q0 += 32) {
    const int nqc = min(32, np - q0);
    __syncthreads();  // Ms visible; f (and mls) free
    if (np > 32) {    // the first pass left only the last chunk in mls
      load_ml(q0, nqc);
      __syncthreads();
    }
    for (int i = d; i < nqc * NQP; i += kHeadDim) {
      const int q = i / NQP, c = i - q * NQP;
      f[q][c] = ex2(mls[q][c].x - Ms[c]);
    }
    __syncthreads();
    if (d < NQP)
      for (int q = 0; q < nqc; ++q) L += mls[q][d].y * f[q][d];
    // row d of O, pieces in order, four pieces' loads in flight together
    for (int q = 0; q < nqc; q += 4) {
      float4 v[4][NQP / 4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (q + i < nqc) {
          const float4* row =
              reinterpret_cast<const float4*>(po + (static_cast<int64_t>(q0 + q + i) * kHeadDim + d) * NQP);
#pragma unroll
          for (int c4 = 0; c4 < NQP / 4; ++c4) v[i][c4] = __ldcg(row + c4);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (q + i < nqc) {
#pragma unroll
          for (int c4 = 0; c4 < NQP / 4; ++c4) {
            acc[4 * c4 + 0] += f[q + i][4 * c4 + 0] * v[i][c4].x;
            acc[4 * c4 + 1] += f[q + i][4 * c4 + 1] * v[i][c4].y;
            acc[4 * c4 + 2] += f[q + i][4 * c4 + 2] * v[i][c4].z;
            acc[4 * c4 + 3] += f[q + i][4 * c4 + 3] * v[i][c4].w;
          }
        }
      }
    }
  }
  if (d < NQP) Linv[d] = L > 0.f ? 1.f / L : 0.f;
  __syncthreads();
  T* optr = static_cast<T*>(p.out);
#pragma unroll
  for (int c = 0; c < NQP; ++c) {
    if (c >= p.nq) break;
    const int qi = c / p.group, gi = c - qi * p.group;
    optr[((static_cast<int64_t>(b) * p.q_len + qi) * p.num_q_heads + h * p.group + gi) * kHeadDim + d] =
        from_f32<T>(acc[c] * Linv[c]);
  }
  if (p.num_peers > 0) {
    __syncthreads();
    copy_segment_to_peers<T>(p, optr, b, h, d, kHeadDim);
  }
  if (d == 0) p.counters[seg_id] = 0;
}

// ------------------------------------------------------------------ generic path
struct GenericParams {
  void* out;
  const void* query;
  const void* key;    // pool base (or contiguous K)
  const void* value;  // pool base (or contiguous V)
  int64_t s_blk, s_head, s_tok;  // element strides of block, kv head, token-in-block
  int32_t block_size;
  const void* block_tables;  // nullptr: block index = token / block_size (contiguous K/V)
  int32_t bt_bytes;
  int64_t bt_stride;
  const int32_t* context_lens;
  int32_t max_context_len;
  int32_t q_len, num_q_heads, num_kv_heads, head_dim;
  int64_t num_blocks;
  float scale;
  int32_t* error_word;
};

constexpr int kGenThreads = 128;
constexpr int kGenMaxDim = 512;

// One CTA per (query row, sequence): fp32 online softmax over the visible keys.
template <typename T>
__global__ void __launch_bounds__(kGenThreads) attn_generic_kernel(const GenericParams p) {
  __shared__ float qs[kGenMaxDim];
  __shared__ float ps[kGenThreads];
  __shared__ int64_t rowoff[kGenThreads];
  __shared__ float red[kGenThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r = blockIdx.x;  // qi * Hq + hq
  const int b = blockIdx.y;
  const int qi = r / p.num_q_heads, hq = r - qi * p.num_q_heads;
  const int group = p.num_q_heads / p.num_kv_heads;
  const int h = hq / group;
  const int D = p.head_dim;

  int64_t L = p.context_lens != nullptr ? p.context_lens[b] : p.max_context_len;
  if (L < 0) L = 0;
  if (p.block_tables != nullptr && L > p.bt_stride * p.block_size) {
    if (tid == 0) report_error(p.error_word, INFERD_ERR_DEVICE_INDEX);
    L = p.bt_stride * p.block_size;
  }
  const int64_t limit = L - p.q_len + qi;  // last visible key position
  const int64_t nvis = limit + 1 < L ? (limit + 1 > 0 ? limit + 1 : 0) : L;

  const T* q = static_cast<const T*>(p.query) + ((static_cast<int64_t>(b) * p.q_len + qi) * p.num_q_heads + hq) * D;
  for (int d = tid; d < D; d += kGenThreads) qs[d] = to_f32<T>(q[d]) * p.scale;
  __syncthreads();

  const T* K = static_cast<const T*>(p.key);
  const T* V = static_cast<const T*>(p.value);
  float acc[kGenMaxDim / kGenThreads];
#pragma unroll
  for (int i = 0; i < kGenMaxDim / kGenThreads; ++i) acc[i] = 0.f;
  float m = -INFINITY, lsum = 0.f;

  for (int64_t t0 = 0; t0 < nvis; t0 += kGenThreads) {
    const int64_t t = t0 + tid;
    float s = -INFINITY;
    int64_t off = -1;
    if (t < nvis) {
      const int64_t page = t / p.block_size;
      const int64_t in = t - page * p.block_size;
      int64_t blk = page;
      if (p.block_tables != nullptr) {
        const int64_t i = static_cast<int64_t>(b) * p.bt_stride + page;
        blk = p.bt_bytes == 8 ? static_cast<const int64_t*>(p.block_tables)[i]
                              : static_cast<int64_t>(static_cast<const int32_t*>(p.block_tables)[i]);
      }
      if (blk < 0 || blk >= p.num_blocks) {
        report_error(p.error_word, INFERD_ERR_DEVICE_INDEX);
      } else {
        off = blk * p.s_blk + h * p.s_head + in * p.s_tok;
        float acc_s = 0.f;
        for (int d = 0; d < D; ++d) acc_s += qs[d] * to_f32<T>(K[off + d]);
        s = acc_s;
      }
    }
    rowoff[tid] = off;
    // block max
    float mx = s;
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < kGenThreads / 32; ++w) mx = fmaxf(mx, red[w]);
    const float mnew = fmaxf(m, mx);
    const float mref = mnew == -INFINITY ? 0.f : mnew;
    const float alpha = expf(m - mref);
    const float pv = (off >= 0) ? expf(s - mref) : 0.f;
    ps[tid] = pv;
    __syncthreads();  // red reuse + ps visible
    float sum = pv;
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) red[warp] = sum;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < kGenThreads / 32; ++w) tot += red[w];
    lsum = lsum * alpha + tot;
    m = mnew;
    const int n = static_cast<int>(min64(kGenThreads, nvis - t0));
#pragma unroll
    for (int i = 0; i < kGenMaxDim / kGenThreads; ++i) {
      const int d = tid + i * kGenThreads;
      if (d < D) {
        float a = acc[i] * alpha;
        for (int j = 0; j < n; ++j) {
          const int64_t ro = rowoff[j];
          if (ro >= 0) a += ps[j] * to_f32<T>(V[ro + d]);
        }
        acc[i] = a;
      }
    }
    __syncthreads();  // before rowoff / ps / red are overwritten
  }
  T* out = static_cast<T*>(p.out) + ((static_cast<int64_t>(b) * p.q_len + qi) * p.num_q_heads + hq) * D;
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
#pragma unroll
  for (int i = 0; i < kGenMaxDim / kGenThreads; ++i) {
    const int d = tid + i * kGenThreads;
    if (d < D) out[d] = from_f32<T>(acc[i] * inv);
  }
}

int launch_generic(const GenericParams& gp, int32_t dtype, int32_t num_seqs, cudaStream_t s) {
  dim3 grid(gp.q_len * gp.num_q_heads, num_seqs);
  if (dtype == INFERD_F32) attn_generic_kernel<float><<<grid, kGenThreads, 0, s>>>(gp);
  else if (dtype == INFERD_F16) attn_generic_kernel<__half><<<grid, kGenThreads, 0, s>>>(gp);
  else attn_generic_kernel<__nv_bfloat16><<<grid, kGenThreads, 0, s>>>(gp);
  return launch_status();
}

// ------------------------------------------------------------------ fast-path host side
inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }


struct WorkspaceLayout {
  size_t counters, ml, o, total;
};

// Workspace: [ticket counters: fixed kCounterRegionBytes][partial (m, l)][partial O].
// The counter region has the same size for every call, so calls of different shapes can
// share one workspace: partials of one call never land on another call's counters, and
// every completed call leaves the counters it used at zero.
constexpr size_t kCounterRegionBytes =
    static_cast<size_t>(kMaxSeqsFast) * kMaxKvHeadsFast * sizeof(int32_t);

inline WorkspaceLayout workspace_layout(int num_seqs, int num_kv_heads, int nqp, int grid) {
  WorkspaceLayout w;
  const size_t segs = static_cast<size_t>(num_seqs) * num_kv_heads;
  // one partial slot per (warp unit, segment) index pair that can occur
  const size_t slots = static_cast<size_t>(grid) * kWarps + segs;
  w.counters = 0;
  w.ml = kCounterRegionBytes;
  w.o = w.ml + align256(slots * nqp * 2 * sizeof(float));
  w.total = w.o + align256(slots * nqp * kHeadDim * sizeof(float));
  return w;
}

inline int fast_grid(int sm_count) { return sm_count * kCtasPerSm; }

// SMs that persistent grids leave free for a collective beside them (process-wide)
std::atomic<int> g_reserved_sms{0};

// SMs the persistent grid of a call launched now may fill
inline int grid_sms() {
  const int sms = current_sm_count();
  const int r = g_reserved_sms.load(std::memory_order_relaxed);
  return r < sms ? sms - r : 1;
}

inline size_t fast_smem_bytes(int num_seqs) {
  return 1024 + static_cast<size_t>(kWarps) * kStagesPerWarp * (kStageBytes + 8) +
         (static_cast<size_t>(num_seqs) + 1) * 4;
}

// Tensor map over one pool viewed as [num_blocks * num_kv_heads * 16 rows, 128 elements]
// with a 64 x 16 box (128 B rows) and 128-byte swizzle.
struct MapCache {
  std::mutex mu;
  struct Entry {
    const void* ptr;
    int64_t rows;
    int dev;
    CUtensorMap map;
  } e[16];
  int n = 0, next = 0;
};
MapCache g_maps;

int pool_map(const void* pool, int64_t rows, CUtensorMap* out) {
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lock(g_maps.mu);
    for (int i = 0; i < g_maps.n; ++i)
      if (g_maps.e[i].ptr == pool && g_maps.e[i].rows == rows && g_maps.e[i].dev == dev) {
        *out = g_maps.e[i].map;
        return INFERD_OK;
      }
  }
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return INFERD_ERR_CUDA;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(kHeadDim * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(kPage)};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMap map;
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(pool), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return INFERD_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_maps.mu);
  MapCache::Entry& e = g_maps.e[g_maps.next];
  e.ptr = pool;
  e.rows = rows;
  e.dev = dev;
  e.map = map;
  g_maps.next = (g_maps.next + 1) % 16;
  if (g_maps.n < 16) ++g_maps.n;
  *out = map;
  return INFERD_OK;
}

template <bool kBf16, int NT, int STAGES = kStagesPerWarp>
int launch_fast_t(const CUtensorMap& km, const CUtensorMap& vm, const FastParams& fp, int grid,
                  size_t smem, cudaStream_t s) {
  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(paged_attn_tc_kernel<kBf16, NT, STAGES>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return cuda_status(e);
    // all of the unified L1/shared array as shared memory, so two CTAs fit per SM
    e = cudaFuncSetAttribute(paged_attn_tc_kernel<kBf16, NT, STAGES>,
                             cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e);
    configured[dev] = true;
  }
  paged_attn_tc_kernel<kBf16, NT, STAGES><<<grid, kWarps * 32, smem, s>>>(km, vm, fp);
  return launch_status();
}

template <bool kBf16>
int launch_fast(const CUtensorMap& km, const CUtensorMap& vm, const FastParams& fp, int nt,
                int grid, size_t smem, cudaStream_t s) {
  switch (nt) {
    case 1: return launch_fast_t<kBf16, 1>(km, vm, fp, grid, smem, s);
    case 2: return launch_fast_t<kBf16, 2>(km, vm, fp, grid, smem, s);
    case 3: return launch_fast_t<kBf16, 3>(km, vm, fp, grid, smem, s);
    default: return launch_fast_t<kBf16, 4>(km, vm, fp, grid, smem, s);
  }
}

template <bool kBf16, int NQP>
int launch_merge_t(const FastParams& fp, int segs, cudaStream_t s) {
  using T = typename std::conditional<kBf16, __nv_bfloat16, __half>::type;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(segs));
  cfg.blockDim = dim3(kHeadDim);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, merge_cut_segments_kernel<T, NQP>, fp));
}

template <bool kBf16>
int launch_merge(const FastParams& fp, int nt, int segs, cudaStream_t s) {
  switch (nt) {
    case 1: return launch_merge_t<kBf16, 8>(fp, segs, s);
    case 2: return launch_merge_t<kBf16, 16>(fp, segs, s);
    case 3: return launch_merge_t<kBf16, 24>(fp, segs, s);
    default: return launch_merge_t<kBf16, 32>(fp, segs, s);
  }
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

}  // namespace

bool paged_attention_fast_path(int32_t dtype, int32_t head_dim, int32_t block_size, int32_t nq,
                               int64_t num_blocks, int32_t num_kv_heads, const void* key_cache,
                               const void* value_cache, const void* query, const void* out) {
  const int64_t rows = num_blocks * num_kv_heads * kPage;
  return (dtype == INFERD_BF16 || dtype == INFERD_F16) && head_dim == kHeadDim &&
         block_size == kPage && nq <= kMaxRowsFast && rows < (int64_t{1} << 31) &&
         num_kv_heads <= kMaxKvHeadsFast && aligned(key_cache, 16) && aligned(value_cache, 16) &&
         aligned(query, 16) && aligned(out, 16);
}

}  // namespace inferd

using namespace inferd;

extern "C" int inferd_paged_attention_reserve_sms(int32_t sms) {
  if (sms < 0 || sms >= current_sm_count()) return INFERD_ERR_INVALID_ARGUMENT;
  g_reserved_sms.store(sms, std::memory_order_relaxed);
  return INFERD_OK;
}

extern "C" int32_t inferd_paged_attention_reserved_sms(void) {
  return g_reserved_sms.load(std::memory_order_relaxed);
}

extern "C" size_t inferd_paged_attention_counter_bytes(int32_t num_seqs, int32_t num_kv_heads) {
  if (num_seqs <= 0 || num_kv_heads <= 0) return 0;
  const size_t seqs = num_seqs < kMaxSeqsFast ? num_seqs : kMaxSeqsFast;
  return align256(seqs * num_kv_heads * sizeof(int32_t));
}

extern "C" size_t inferd_paged_attention_workspace_bytes(int32_t num_seqs, int32_t q_len,
                                                         int32_t num_q_heads, int32_t num_kv_heads,
                                                         int32_t head_dim, int32_t device) {
  if (num_seqs <= 0 || q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return 0;
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      sms <= 0) {
    cudaGetLastError();
    sms = 148;
  }
  const int group = num_q_heads / (num_kv_heads > 0 ? num_kv_heads : 1);
  const int nqp = nq_pad(q_len * (group > 0 ? group : 1));
  const int chunk = num_seqs < kMaxSeqsFast ? num_seqs : kMaxSeqsFast;
  return workspace_layout(chunk, num_kv_heads, nqp, fast_grid(sms)).total;
}

static int paged_attention_impl(void* out, const void* query, const void* key_cache,
                                const void* value_cache, const void* block_tables,
                                int32_t block_table_bytes, int64_t block_table_stride,
                                const int32_t* context_lens, int32_t num_seqs, int32_t q_len,
                                int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                int32_t block_size, int64_t num_blocks, int32_t max_context_len,
                                float scale, int32_t dtype, void* workspace,
                                size_t workspace_bytes, int32_t* error_word, void* stream,
                                void* const* peer_out, int32_t num_peers, int64_t peer_offset) {
  if (num_seqs < 0 || q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || num_blocks <= 0 || max_context_len < 0 || block_table_stride < 0)
    return INFERD_ERR_INVALID_ARGUMENT;
  if (num_q_heads % num_kv_heads != 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (block_table_bytes != 4 && block_table_bytes != 8) return INFERD_ERR_INVALID_ARGUMENT;
  if (dtype != INFERD_F32 && dtype != INFERD_F16 && dtype != INFERD_BF16)
    return INFERD_ERR_UNSUPPORTED;
  if (num_seqs == 0) return INFERD_OK;
  if (!out || !query || !key_cache || !value_cache || !block_tables)
    return INFERD_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int group = num_q_heads / num_kv_heads;
  const int nq = q_len * group;
  const int64_t rows = num_blocks * num_kv_heads * kPage;

  const bool fast = paged_attention_fast_path(dtype, head_dim, block_size, nq, num_blocks,
                                              num_kv_heads, key_cache, value_cache, query, out);
  if (!fast) {
    if (num_peers > 0) return INFERD_ERR_UNSUPPORTED;  // the gathered form is the fast path's
    if (head_dim > kGenMaxDim) return INFERD_ERR_UNSUPPORTED;
    if (static_cast<int64_t>(q_len) * num_q_heads > 65535 * 1024) return INFERD_ERR_UNSUPPORTED;
    GenericParams gp;
    gp.out = out;
    gp.query = query;
    gp.key = key_cache;
    gp.value = value_cache;
    gp.s_tok = head_dim;
    gp.s_head = static_cast<int64_t>(block_size) * head_dim;
    gp.s_blk = static_cast<int64_t>(num_kv_heads) * block_size * head_dim;
    gp.block_size = block_size;
    gp.block_tables = block_tables;
    gp.bt_bytes = block_table_bytes;
    gp.bt_stride = block_table_stride;
    gp.context_lens = context_lens;
    gp.max_context_len = max_context_len;
    gp.q_len = q_len;
    gp.num_q_heads = num_q_heads;
    gp.num_kv_heads = num_kv_heads;
    gp.head_dim = head_dim;
    gp.num_blocks = num_blocks;
    gp.scale = scale;
    gp.error_word = error_word;
    // gridDim.y is limited to 65535 sequences per launch
    for (int32_t b0 = 0; b0 < num_seqs; b0 += 65535) {
      const int32_t nb = num_seqs - b0 < 65535 ? num_seqs - b0 : 65535;
      GenericParams g2 = gp;
      const int es = dtype_bytes(dtype);
      g2.out = static_cast<uint8_t*>(out) + static_cast<int64_t>(b0) * q_len * num_q_heads * head_dim * es;
      g2.query = static_cast<const uint8_t*>(query) + static_cast<int64_t>(b0) * q_len * num_q_heads * head_dim * es;
      g2.block_tables = static_cast<const uint8_t*>(block_tables) + b0 * block_table_stride * block_table_bytes;
      g2.context_lens = context_lens ? context_lens + b0 : nullptr;
      const int st = launch_generic(g2, dtype, nb, s);
      if (st != INFERD_OK) return st;
    }
    return INFERD_OK;
  }

  const int nqp = nq_pad(nq);
  const int grid = fast_grid(grid_sms());
  // the cut-segment marker of the merge kernel packs a piece count below 2^11
  if (nqp > 8 && grid * kWarps >= (1 << 11)) return INFERD_ERR_UNSUPPORTED;
  const int chunk_max = kMaxSeqsFast;
  const WorkspaceLayout wl = workspace_layout(num_seqs < chunk_max ? num_seqs : chunk_max,
                                              num_kv_heads, nqp, grid);
  if (workspace == nullptr || !aligned(workspace, 256) || workspace_bytes < wl.total)
    return INFERD_ERR_WORKSPACE;

  CUtensorMap km, vm;
  int st = pool_map(key_cache, rows, &km);
  if (st != INFERD_OK) return st;
  st = pool_map(value_cache, rows, &vm);
  if (st != INFERD_OK) return st;

  const int es = dtype_bytes(dtype);
  for (int32_t b0 = 0; b0 < num_seqs; b0 += chunk_max) {
    const int32_t nb = num_seqs - b0 < chunk_max ? num_seqs - b0 : chunk_max;
    FastParams fp;
    fp.out = static_cast<uint8_t*>(out) + static_cast<int64_t>(b0) * q_len * num_q_heads * kHeadDim * es;
    fp.query = static_cast<const uint8_t*>(query) + static_cast<int64_t>(b0) * q_len * num_q_heads * kHeadDim * es;
    fp.block_tables = static_cast<const uint8_t*>(block_tables) + b0 * block_table_stride * block_table_bytes;
    fp.bt_stride = block_table_stride;
    fp.bt_bytes = block_table_bytes;
    fp.context_lens = context_lens ? context_lens + b0 : nullptr;
    fp.max_context_len = max_context_len;
    fp.num_seqs = nb;
    fp.q_len = q_len;
    fp.num_q_heads = num_q_heads;
    fp.num_kv_heads = num_kv_heads;
    fp.group = group;
    fp.nq = nq;
    fp.num_blocks = num_blocks;
    fp.scale_log2 = scale * kLog2e;
    fp.counters = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + wl.counters);
    fp.part_ml = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + wl.ml);
    fp.part_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + wl.o);
    fp.error_word = error_word;
    fp.peer_out = peer_out;
    fp.num_peers = num_peers;
    fp.peer_offset = peer_offset + static_cast<int64_t>(b0) * q_len * num_q_heads * kHeadDim;
    // Several n-tiles: the kernel leaves the partials of cut segments to a second, fully
    // parallel kernel (merge_cut_segments_kernel)
    const bool defer_merge = nqp > 8;
    // grid: persistent, but no more CTAs than pages can feed (upper bound from the host)
    const int64_t pages_ub = static_cast<int64_t>(nb) * num_kv_heads *
                             ((static_cast<int64_t>(max_context_len) + kPage - 1) / kPage);
    int g = grid;
    const int64_t ctas_ub = (pages_ub + kWarps - 1) / kWarps;  // one warp per page at most
    if (ctas_ub < g) g = ctas_ub > 0 ? static_cast<int>(ctas_ub) : 1;
    const size_t smem = fast_smem_bytes(nb);
    st = dtype == INFERD_BF16 ? launch_fast<true>(km, vm, fp, nqp / 8, g, smem, s)
                              : launch_fast<false>(km, vm, fp, nqp / 8, g, smem, s);
    if (st != INFERD_OK) return st;
    if (defer_merge) {
      st = dtype == INFERD_BF16 ? launch_merge<true>(fp, nqp / 8, nb * num_kv_heads, s)
                                : launch_merge<false>(fp, nqp / 8, nb * num_kv_heads, s);
      if (st != INFERD_OK) return st;
    }
  }
  return INFERD_OK;
}

extern "C" int inferd_paged_attention(void* out, const void* query, const void* key_cache,
                                      const void* value_cache, const void* block_tables,
                                      int32_t block_table_bytes, int64_t block_table_stride,
                                      const int32_t* context_lens, int32_t num_seqs,
                                      int32_t q_len, int32_t num_q_heads, int32_t num_kv_heads,
                                      int32_t head_dim, int32_t block_size, int64_t num_blocks,
                                      int32_t max_context_len, float scale, int32_t dtype,
                                      void* workspace, size_t workspace_bytes,
                                      int32_t* error_word, void* stream) {
  return paged_attention_impl(out, query, key_cache, value_cache, block_tables, block_table_bytes,
                              block_table_stride, context_lens, num_seqs, q_len, num_q_heads,
                              num_kv_heads, head_dim, block_size, num_blocks, max_context_len,
                              scale, dtype, workspace, workspace_bytes, error_word, stream,
                              nullptr, 0, 0);
}

extern "C" int inferd_paged_attention_gather(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const void* block_tables, int32_t block_table_bytes, int64_t block_table_stride,
    const int32_t* context_lens, int32_t num_seqs, int32_t q_len, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int64_t num_blocks,
    int32_t max_context_len, float scale, int32_t dtype, void* workspace, size_t workspace_bytes,
    void* const* peer_out, int32_t num_peers, int64_t peer_offset, int32_t* error_word,
    void* stream) {
  if (num_peers < 1 || num_peers > 64 || peer_out == nullptr || peer_offset < 0 ||
      peer_offset % 8 != 0)
    return INFERD_ERR_INVALID_ARGUMENT;
  return paged_attention_impl(out, query, key_cache, value_cache, block_tables, block_table_bytes,
                              block_table_stride, context_lens, num_seqs, q_len, num_q_heads,
                              num_kv_heads, head_dim, block_size, num_blocks, max_context_len,
                              scale, dtype, workspace, workspace_bytes, error_word, stream,
                              peer_out, num_peers, peer_offset);
}

extern "C" int inferd_dense_attention(void* out, const void* query, const void* key,
                                      const void* value, int64_t seq_len, int32_t q_len,
                                      int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                                      float scale, int32_t dtype, void* stream) {
  if (seq_len < 0 || q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return INFERD_ERR_INVALID_ARGUMENT;
  if (num_q_heads % num_kv_heads != 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (dtype != INFERD_F32 && dtype != INFERD_F16 && dtype != INFERD_BF16)
    return INFERD_ERR_UNSUPPORTED;
  if (head_dim > kGenMaxDim) return INFERD_ERR_UNSUPPORTED;
  if (seq_len > INT32_MAX) return INFERD_ERR_UNSUPPORTED;
  if (!out || !query || (seq_len > 0 && (!key || !value))) return INFERD_ERR_INVALID_ARGUMENT;
  GenericParams gp;
  gp.out = out;
  gp.query = query;
  gp.key = key;
  gp.value = value;
  gp.s_tok = static_cast<int64_t>(num_kv_heads) * head_dim;
  gp.s_head = head_dim;
  gp.s_blk = 0;
  gp.block_size = seq_len > 0 ? static_cast<int32_t>(seq_len) : 1;
  gp.block_tables = nullptr;
  gp.bt_bytes = 4;
  gp.bt_stride = 1;
  gp.context_lens = nullptr;
  gp.max_context_len = static_cast<int32_t>(seq_len);
  gp.q_len = q_len;
  gp.num_q_heads = num_q_heads;
  gp.num_kv_heads = num_kv_heads;
  gp.head_dim = head_dim;
  gp.num_blocks = 1;
  gp.scale = scale;
  gp.error_word = nullptr;
  return launch_generic(gp, dtype, 1, static_cast<cudaStream_t>(stream));
}
