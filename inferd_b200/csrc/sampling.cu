// sampling.cu -- decode-step sampling on the GPU: temperature + top-p (nucleus)
// probabilities and one multinomial draw per row.
//
// Reference: core/spec_decode.py:14-31 nucleus_probs (softmax(logits / T), descending
// sort, inclusive cumsum, zero entries whose exclusive cumulative mass exceeds top_p,
// renormalise; T <= 0 gives a one-hot row at the argmax) and :34-35 sample_from
// (torch.multinomial, one sample).  Callers: the scheduler's per-request sampling
// (core/scheduler.py:341-342) and the speculative accept/resample loop
// (core/spec_decode.py:127-160).
//
// Layout: one cluster of C CTAs (C = 1, 2, 4 or 8) per row; CTA r holds the row's
// elements [r * per_cta, (r + 1) * per_cta) in shared memory (fp32, at most 32768 per
// CTA), so the logits are read from HBM once and every later pass runs on chip.
// Cluster-wide values (max, sums, histograms) are exchanged through distributed shared
// memory and combined in rank order, so every CTA reaches the same decisions.
//
// No sort: the top-p cut is found by a radix select on the fp32 bit patterns of the
// probabilities (monotonic for p >= 0), four passes of 8 bits with 256-bin histograms of
// count and mass.  Masses are summed as integers (round(p * 2^31) in the select,
// round(p * 2^52) for the draw), so nothing depends on the order of atomic updates.  The kept set is every entry whose exclusive cumulative
// mass in descending order is <= top_p, ties in index order (a stable sort; the
// reference's torch.sort leaves the order of equal values unspecified).
//
// The draw is an inverse CDF in index order over the kept fixed-point masses with 64
// random bits per row from Philox4x32-10 (Salmon et al., SC 2011) keyed by the caller's
// seed, counter = offset + row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <type_traits>

#include "common.cuh"
#include "runtime.cuh"

namespace inferd {
namespace {

constexpr int kSampThreads = 512;
constexpr int kSampWarps = kSampThreads / 32;
constexpr int kSampMaxPerCta = 32768;   // fp32 entries held per CTA (128 KB)
constexpr int kSampChunk = kSampThreads * 8;  // index-ordered passes: 8 consecutive per thread
constexpr double kFixedOne = 4503599627370496.0;  // 2^52

struct SampParams {
  const void* src;       // logits (mode 0) or probabilities (mode 1), [rows, stride]
  int64_t stride;        // elements between rows of src
  int64_t vocab;
  int32_t rows;
  int32_t per_cta;
  int32_t mode;          // 0: nucleus from logits, 1: draw from given probabilities
  const float* temps;    // per-row temperature (nullable: temp)
  float temp;
  const float* top_ps;   // per-row top_p (nullable: top_p)
  float top_p;
  float* probs_out;      // [rows, out_stride] (nullable)
  int64_t out_stride;
  int64_t* tokens;       // [rows] (nullable)
  uint64_t seed, offset;
  int32_t* error_word;
};

// ---------------------------------------------------------------- cluster helpers
__device__ __forceinline__ uint32_t samp_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void samp_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the two halves of samp_cluster_sync, with independent work between them
__device__ __forceinline__ void samp_cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void samp_cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Generic address of this CTA's shared variable *p as seen in CTA `rank` of the cluster.
// Reads through it are ordinary loads, so several can be in flight; the cluster barriers
// (with memory clobbers) order them against the writes they read.
template <typename T>
__device__ __forceinline__ const T* cl_ptr(const T* p, uint32_t rank) {
  unsigned long long r;
  asm volatile("mapa.u64 %0, %1, %2;" : "=l"(r) : "l"(reinterpret_cast<unsigned long long>(p)), "r"(rank));
  return reinterpret_cast<const T*>(r);
}
__device__ __forceinline__ float ld_cl_f32(const float* p, uint32_t rank) { return *cl_ptr(p, rank); }
__device__ __forceinline__ uint32_t ld_cl_u32(const void* p, uint32_t rank) {
  return *cl_ptr(static_cast<const uint32_t*>(p), rank);
}
__device__ __forceinline__ unsigned long long ld_cl_u64(const unsigned long long* p, uint32_t rank) {
  return *cl_ptr(p, rank);
}

// ---------------------------------------------------------------- Philox4x32-10
__device__ __forceinline__ void philox_round(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
  const uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
  const uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
  const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
  c[0] = n0;
  c[1] = lo1;
  c[2] = n2;
  c[3] = lo0;
}
// 64 random bits for counter n under key seed: words 0 (high) and 1 (low) of the block
__device__ __forceinline__ unsigned long long philox_u64(uint64_t seed, uint64_t n) {
  uint32_t c[4] = {static_cast<uint32_t>(n), static_cast<uint32_t>(n >> 32), 0u, 0u};
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    philox_round(c, k0, k1);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return (static_cast<unsigned long long>(c[0]) << 32) | c[1];
}

// round(v * scale) as an integer; scale is a power of two, so the product is exact (short
// of underflow) and only the final rounding happens
__device__ __forceinline__ unsigned long long to_fixed(float v, float scale) {
  return __float2ull_rn(v * scale);
}

template <typename In>
__device__ __forceinline__ float load_src(const In* p) {
  return to_f32<In>(*p);
}

// ---------------------------------------------------------------- block reductions
constexpr int kMaxSweeps = kSampMaxPerCta / kSampThreads;

struct SampShared {
  uint32_t hist_m[2][256];  // select histograms: mass (multiples of 2^-31) and count,
  uint32_t hist_c[2][256];  // double-buffered by pass
  unsigned long long tot_m[256];  // the cluster's sums
  uint32_t tot_c[256];
  uint32_t tie_cnt[kMaxSweeps * kSampWarps];
  float wf[kSampWarps];
  int wi[kSampWarps];
  unsigned long long wu[kSampWarps];
  // values published to the cluster
  float x_f;
  int x_i;
  unsigned long long x_u;
  unsigned long long x_u2;
  // broadcasts
  uint32_t b_prefix;
  unsigned long long b_mass;
  uint32_t b_ties;
  unsigned long long b_u;
  float b_f;
  int b_i;
  int found;
};

// max of (v, idx) with the smaller index on equal values, broadcast to every thread
template <class Sh>
__device__ __forceinline__ void block_argmax(Sh& sh, float& v, int& idx) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  if (lane == 0) {
    sh.wf[w] = v;
    sh.wi[w] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    v = sh.wf[0];
    idx = sh.wi[0];
    for (int k = 1; k < kSampWarps; ++k)
      if (sh.wf[k] > v || (sh.wf[k] == v && sh.wi[k] < idx)) {
        v = sh.wf[k];
        idx = sh.wi[k];
      }
    sh.b_f = v;
    sh.b_i = idx;
  }
  __syncthreads();
  v = sh.b_f;
  idx = sh.b_i;
  __syncthreads();
}

// fp32 sum in a fixed order (xor tree within warps, then warp order), broadcast
template <class Sh>
__device__ __forceinline__ float block_sum_f32(Sh& sh, float v) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) sh.wf[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int k = 0; k < kSampWarps; ++k) s += sh.wf[k];
    sh.b_f = s;
  }
  __syncthreads();
  const float s = sh.b_f;
  __syncthreads();
  return s;
}

template <class Sh>
__device__ __forceinline__ unsigned long long block_sum_u64(Sh& sh, unsigned long long v) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (lane == 0) sh.wu[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long s = 0;
    for (int k = 0; k < kSampWarps; ++k) s += sh.wu[k];
    sh.b_u = s;
  }
  __syncthreads();
  const unsigned long long s = sh.b_u;
  __syncthreads();
  return s;
}

// exclusive prefix of v over the block in thread order, and the block total
template <class Sh>
__device__ __forceinline__ unsigned long long block_exscan_u64(Sh& sh, unsigned long long v,
                                                               unsigned long long& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned long long inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) sh.wu[w] = inc;
  __syncthreads();
  unsigned long long base = 0, tot = 0;
  for (int k = 0; k < kSampWarps; ++k) {
    if (k < w) base += sh.wu[k];
    tot += sh.wu[k];
  }
  __syncthreads();
  total = tot;
  return base + inc - v;
}

// One loaded entry: x / T (mode 0), weight sanity (mode 1), store, running argmax.
__device__ __forceinline__ void take_entry(float* e, int i, float x, int64_t lo, int mode, bool greedy,
                                           float temp, bool& bad, float& mv, int& mi) {
  if (mode == 0 && !greedy) x = __fdiv_rn(x, temp);
  if (mode == 1 && (!(x >= 0.f) || x == INFINITY)) {  // negative, NaN or infinite weight
    bad = true;
    x = 0.f;
  }
  e[i] = x;
  const int gi = static_cast<int>(lo) + i;
  if (x > mv || (x == mv && gi < mi)) {
    mv = x;
    mi = gi;
  }
}

// mass of p in units of 2^-31 for the radix select (p <= 1, so it fits 32 bits)
__device__ __forceinline__ uint32_t to_q31(float p) { return __float2uint_rn(p * 2147483648.0f); }

// ---------------------------------------------------------------- the kernel
// mode 0: probs_out (optional) = nucleus probabilities; tokens (optional) = one draw.
// mode 1: tokens = one draw from the given non-negative weights (sample_from).
template <int C, typename In>
__global__ void __launch_bounds__(kSampThreads) sampling_kernel(const SampParams p) {
  extern __shared__ __align__(16) float e[];
  __shared__ SampShared sh;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const uint32_t rank = samp_rank();
  const int row = blockIdx.x / C;
  const int64_t lo = static_cast<int64_t>(rank) * p.per_cta;
  int n = static_cast<int>(p.vocab - lo < p.per_cta ? p.vocab - lo : p.per_cta);
  if (n < 0) n = 0;
  const In* src = static_cast<const In*>(p.src) + static_cast<int64_t>(row) * p.stride + lo;
  const float temp = p.temps ? p.temps[row] : p.temp;
  const float top_p = p.top_ps ? p.top_ps[row] : p.top_p;
  const bool greedy = p.mode == 0 && !(temp > 0.f);

  // ---- phase 1: load (x / T) and the row max (argmax with the smallest index)
  float mv = -INFINITY;
  int mi = 0x7fffffff;
  bool bad = false;
  {
    constexpr int kVec = 16 / static_cast<int>(sizeof(In));
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const int nv = n / kVec;
      const uint4* src4 = reinterpret_cast<const uint4*>(src);
#pragma unroll 8
      for (int v = tid; v < nv; v += kSampThreads) {
        const uint4 raw = __ldg(src4 + v);
        const In* el = reinterpret_cast<const In*>(&raw);
#pragma unroll
        for (int j = 0; j < kVec; ++j)
          take_entry(e, v * kVec + j, to_f32<In>(el[j]), lo, p.mode, greedy, temp, bad, mv, mi);
      }
      done = nv * kVec;
    }
    for (int i = done + tid; i < n; i += kSampThreads)
      take_entry(e, i, load_src<In>(src + i), lo, p.mode, greedy, temp, bad, mv, mi);
  }
  if (bad) report_error(p.error_word, INFERD_ERR_INVALID_ARGUMENT);
  block_argmax(sh, mv, mi);
  if (tid == 0) {
    sh.x_f = mv;
    sh.x_i = mi;
  }
  samp_cluster_sync();
  float gmax = -INFINITY;
  int gidx = 0x7fffffff;
#pragma unroll
  for (int r = 0; r < C; ++r) {
    const float v = ld_cl_f32(&sh.x_f, r);
    const int ix = static_cast<int>(ld_cl_u32(&sh.x_i, r));
    if (v > gmax || (v == gmax && ix < gidx)) {
      gmax = v;
      gidx = ix;
    }
  }
  samp_cluster_sync();  // slots are rewritten below

  float* out = p.probs_out ? p.probs_out + static_cast<int64_t>(row) * p.out_stride + lo : nullptr;
  if (greedy) {
    // T <= 0: one-hot at the argmax (core/spec_decode.py:18-21)
    if (out)
      for (int i = tid; i < n; i += kSampThreads) out[i] = (static_cast<int>(lo) + i == gidx) ? 1.f : 0.f;
    if (p.tokens && rank == 0 && tid == 0) p.tokens[row] = gidx;
    return;
  }

  // ---- phase 2: probabilities (mode 0); weights stay as given (mode 1)
  // Fixed point for the draw: probabilities as multiples of 2^-52; weights scaled by the
  // power of two 2^(52 - k) with 2^k >= vocab * max weight, so totals stay <= 2^52.
  float fxs = 4503599627370496.0f;
  if (p.mode == 0) {
    float s = 0.f;
    for (int i = tid; i < n; i += kSampThreads) {
      const float ex = expf(e[i] - gmax);
      e[i] = ex;
      s += ex;
    }
    s = block_sum_f32(sh, s);
    if (tid == 0) sh.x_f = s;
    samp_cluster_sync();
    float z = 0.f;
#pragma unroll
    for (int r = 0; r < C; ++r) z += ld_cl_f32(&sh.x_f, r);
    samp_cluster_sync();
    for (int i = tid; i < n; i += kSampThreads) e[i] = __fdiv_rn(e[i], z);
  } else {
    int ex = 0;
    frexpf(gmax, &ex);  // gmax <= 2^ex (gmax = 0 gives ex = 0)
    const int lv = p.vocab > 1 ? 64 - __clzll(static_cast<unsigned long long>(p.vocab - 1)) : 0;
    int k = ex + lv;
    if (k < 0) k = 0;
    fxs = ldexpf(1.f, 52 - k);
  }

  // ---- phase 3: top-p threshold by radix select on the bits of p
  // The select sums masses as multiples of 2^-31 in 32-bit counters (native shared-memory
  // atomics; a bin's sum is at most the row's total, about 2^31).  An entry is kept when
  // the mass of the entries before it in descending order (ties in index order) is
  // <= round(top_p * 2^31).
  const bool cut = p.mode == 0 && top_p < 1.f;
  uint32_t tbits = 0;
  if (cut) {
    const unsigned long long limit = __double2ull_rn(static_cast<double>(top_p) * 2147483648.0);
    uint32_t prefix = 0;
    unsigned long long above = 0;
    uint32_t ties = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      // a pass's histogram buffer is next written two passes later, after the next pass's
      // cluster barrier, by which time every CTA has read it
      uint32_t* hm = sh.hist_m[(shift >> 3) & 1];
      uint32_t* hc = sh.hist_c[(shift >> 3) & 1];
      for (int b = tid; b < 256; b += kSampThreads) {
        hm[b] = 0;
        hc[b] = 0;
      }
      __syncthreads();
      const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = tid; i < n; i += kSampThreads) {
        const uint32_t bits = __float_as_uint(e[i]);
        if ((bits & hi_mask) == (prefix & hi_mask)) {
          const uint32_t d = (bits >> shift) & 255u;
          atomicAdd(&hm[d], to_q31(e[i]));
          atomicAdd(&hc[d], 1u);
        }
      }
      __syncthreads();
      samp_cluster_sync();  // every CTA's histogram is complete
      for (int b = tid; b < 256; b += kSampThreads) {
        unsigned long long m = 0;
        uint32_t c = 0;
#pragma unroll
        for (int r = 0; r < C; ++r) {
          m += ld_cl_u32(&hm[b], r);
          c += ld_cl_u32(&hc[b], r);
        }
        sh.tot_m[b] = m;
        sh.tot_c[b] = c;
      }
      __syncthreads();
      if (tid < 32) {
        // Lane l owns bins 255 - 8l .. 248 - 8l (descending).  The cut bin is the lowest
        // non-empty bin whose mass above (above + all higher bins) is within the limit.
        unsigned long long mine = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) mine += sh.tot_m[255 - 8 * lane - j];
        unsigned long long pre = mine;  // inclusive scan in lane order
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned long long t = __shfl_up_sync(0xffffffffu, pre, o);
          if (lane >= o) pre += t;
        }
        unsigned long long acc = above + pre - mine;
        int cand = 256;
        unsigned long long cand_acc = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int b = 255 - 8 * lane - j;
          if (sh.tot_c[b] > 0 && acc <= limit) {
            cand = b;
            cand_acc = acc;
          }
          acc += sh.tot_m[b];
        }
        int best = cand;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (best == 256) best = 0;  // not reached: the largest entry always qualifies
        const uint32_t owner = static_cast<uint32_t>((255 - best) / 8);
        const unsigned long long best_acc = __shfl_sync(0xffffffffu, cand_acc, owner);
        if (lane == 0) {
          sh.b_prefix = prefix | (static_cast<uint32_t>(best) << shift);
          sh.b_mass = best_acc;
          sh.b_ties = sh.tot_c[best];
        }
      }
      __syncthreads();
      prefix = sh.b_prefix;
      above = sh.b_mass;
      ties = sh.b_ties;
      __syncthreads();
    }
    tbits = prefix;
    const unsigned long long tq = to_q31(__uint_as_float(tbits));
    uint32_t keep_ties = ties;
    if (tq > 0) {
      const unsigned long long room = (limit - above) / tq + 1;  // above <= limit
      if (room < keep_ties) keep_ties = static_cast<uint32_t>(room);
    }

    // ---- phase 4: a tied group cut in the middle keeps its first entries in index order.
    // Entry i = k * 512 + tid is the k-th sweep's; ranks come from per-(sweep, warp) ballot
    // counts scanned once.
    if (keep_ties < ties) {
      const int nk = (n + kSampThreads - 1) / kSampThreads;  // <= kMaxSweeps
      const int w = tid >> 5;
      for (int k = 0; k < nk; ++k) {
        const int i = k * kSampThreads + tid;
        const bool tie = i < n && __float_as_uint(e[i]) == tbits;
        const uint32_t bal = __ballot_sync(0xffffffffu, tie);
        if (lane == 0) sh.tie_cnt[k * kSampWarps + w] = static_cast<uint32_t>(__popc(bal));
      }
      __syncthreads();
      // exclusive scan of the nk * 16 counts in (sweep, warp) order; thread t owns 2 slots
      const int slots = nk * kSampWarps;
      const uint32_t a0 = 2 * tid < slots ? sh.tie_cnt[2 * tid] : 0u;
      const uint32_t a1 = 2 * tid + 1 < slots ? sh.tie_cnt[2 * tid + 1] : 0u;
      unsigned long long cta_ties;
      const unsigned long long ex = block_exscan_u64(sh, a0 + a1, cta_ties);
      if (2 * tid < slots) sh.tie_cnt[2 * tid] = static_cast<uint32_t>(ex);
      if (2 * tid + 1 < slots) sh.tie_cnt[2 * tid + 1] = static_cast<uint32_t>(ex + a0);
      if (tid == 0) sh.x_u2 = cta_ties;
      samp_cluster_sync();
      unsigned long long base = 0;
      for (uint32_t r = 0; r < rank; ++r) base += ld_cl_u64(&sh.x_u2, r);
      samp_cluster_sync();
      if (base + cta_ties > keep_ties) {  // otherwise every tie of this CTA is kept
        const uint32_t lt = (1u << lane) - 1u;
        for (int k = 0; k < nk; ++k) {
          const int i = k * kSampThreads + tid;
          const bool tie = i < n && __float_as_uint(e[i]) == tbits;
          const uint32_t bal = __ballot_sync(0xffffffffu, tie);
          if (tie) {
            const unsigned long long rk = base + sh.tie_cnt[k * kSampWarps + w] + __popc(bal & lt);
            if (rk >= keep_ties) e[i] = 0.f;  // dropped: excluded below as p < t
          }
        }
      }
      __syncthreads();
    }
  }

  // ---- kept mass in fixed point: this CTA's share, the shares before it, the row total
  unsigned long long local = 0;
  for (int i = tid; i < n; i += kSampThreads) {
    const float v = e[i];
    if (!cut || __float_as_uint(v) >= tbits) local += to_fixed(v, fxs);
  }
  local = block_sum_u64(sh, local);
  if (tid == 0) sh.x_u2 = local;
  samp_cluster_sync();
  unsigned long long base = 0, kept = 0;
#pragma unroll
  for (int r = 0; r < C; ++r) {
    const unsigned long long v = ld_cl_u64(&sh.x_u2, r);
    if (r < static_cast<int>(rank)) base += v;
    kept += v;
  }
  samp_cluster_sync();

  // ---- phase 5: renormalised probabilities
  if (p.mode == 0 && out) {
    const float s = static_cast<float>(static_cast<double>(kept) / kFixedOne);
    auto val = [&](float v) { return ((!cut || __float_as_uint(v) >= tbits) && v > 0.f) ? __fdiv_rn(v, s) : 0.f; };
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      const int nv = n / 4;
      float4* out4 = reinterpret_cast<float4*>(out);
      const float4* e4 = reinterpret_cast<const float4*>(e);
      for (int v = tid; v < nv; v += kSampThreads) {
        const float4 x = e4[v];
        out4[v] = make_float4(val(x.x), val(x.y), val(x.z), val(x.w));
      }
      done = nv * 4;
    }
    for (int i = done + tid; i < n; i += kSampThreads) out[i] = val(e[i]);
  }

  // ---- phase 6: one draw, inverse CDF in index order over the kept masses
  if (p.tokens) {
    if (kept == 0) {
      if (rank == 0 && tid == 0) {
        p.tokens[row] = -1;
        report_error(p.error_word, INFERD_ERR_INVALID_ARGUMENT);
      }
      return;
    }
    const unsigned long long target = __umul64hi(philox_u64(p.seed, p.offset + static_cast<uint64_t>(row)), kept);
    if (target >= base && target < base + local) {
      if (tid == 0) sh.found = 0;
      __syncthreads();
      unsigned long long acc0 = base;
      for (int c0 = 0; c0 < n; c0 += kSampChunk) {
        const int i0 = c0 + tid * 8;
        unsigned long long q[8];
        unsigned long long mine = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          q[j] = 0;
          if (i0 + j < n) {
            const float v = e[i0 + j];
            if (!cut || __float_as_uint(v) >= tbits) q[j] = to_fixed(v, fxs);
          }
          mine += q[j];
        }
        unsigned long long tot_chunk;
        const unsigned long long ex = acc0 + block_exscan_u64(sh, mine, tot_chunk);
        if (target >= ex && target < ex + mine) {
          unsigned long long acc = ex;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc += q[j];
            if (acc > target) {
              p.tokens[row] = lo + i0 + j;
              sh.found = 1;
              break;
            }
          }
        }
        acc0 += tot_chunk;
        __syncthreads();
        if (sh.found) break;
      }
    }
  }
}

// ---------------------------------------------------------------- 16-bit logits (bf16 / f16)
// The same nucleus rule for 16-bit logits with far less on-chip work.  A cluster of C CTAs
// holds a row's raw 16-bit logits in shared memory (half the bytes of fp32 probabilities, so
// a batch of rows fits the GPU in one wave) and recomputes p(x) from them where needed:
//     p(x) = fdiv(expf(fdiv(x, T) - ymax), z)      (the same operations as sampling_kernel)
//
// Candidates.  Only entries with p >= p_min can be kept, where p_min follows from top_p and
// the vocabulary size: with q = round(p * 2^31), the last kept entry j* has every entry from
// j* on (in descending order) at q <= q_j*, and those carry the mass Q - excl(j*) >= Q - L
// (Q the total, L = round(top_p * 2^31)), so V * q_j* >= Q - L; the sum of the rounded p is
// at least 1 - 2^-12 (it is 1 up to the fp32 rounding of z and of each p), so
//     q_j* >= (2^31 (1 - 2^-12) - V / 2 - L) / V.
// Entries below p_min come after every kept entry in the order, so they change neither the
// cut nor any kept entry's exclusive mass: the select, the tie cut, the kept mass and the
// draw need only the candidates.  A candidate test on x itself (x >= thr, thr from p_min
// with a margin far above the rounding of fdiv and expf) lets the candidate pass skip every
// other entry without computing p; each candidate's exact p goes into a per-CTA list in
// index order.  Rows whose candidates overflow a list, and rows with top_p >= 1, take the
// full path: the same steps over every entry, p recomputed in each pass.
constexpr int kN16Threads = 512;
constexpr int kN16CtasPerSm = 2;
constexpr int kN16MaxPerCta = 38912 * 2 / kN16CtasPerSm;  // 16-bit logits per CTA (76 KB at 2 / SM)
constexpr int kN16ListCap = 4096 * 2 / kN16CtasPerSm;  // candidates per CTA: local index + p (f32)
// local index of a candidate: 16 bits while a CTA's slice fits them
using N16Idx = std::conditional<(kN16MaxPerCta > 65536), uint32_t, uint16_t>::type;
constexpr int kN16Chunk = kN16Threads * 8;  // index-ordered passes: 8 consecutive per thread
static_assert(kN16Threads / 32 == kSampWarps, "the block reductions assume 16 warps");

constexpr int kN16Fin = 64;  // entries the select finishes by sorting (cluster-wide)

struct N16Shared {
  __align__(16) uint32_t hist_m[2][256];
  __align__(16) uint32_t hist_c[2][256];
  float wf[kSampWarps];
  int wi[kSampWarps];
  unsigned long long wu[kSampWarps];
  // values published to the cluster (an exchange with a slot of its own, written once,
  // needs one cluster barrier; the kernel's last barrier keeps every CTA alive until the
  // others have read its slots)
  float x_f;
  int x_i;
  unsigned long long x_u;
  float x_mz[2];              // block max of the logits, block sum z relative to it
  unsigned long long x_kept;  // kept mass of the CTA
  // the CTA's entries sharing the threshold's 16-bit prefix (finish of the select)
  uint32_t fin_bits[kN16Fin];
  int fin_idx[kN16Fin];
  int fin_n;
  // their cluster-wide order (warp 0 of each CTA)
  unsigned long long fin_key[kN16Fin];
  uint32_t fin_cut_bits;
  int fin_cut_idx;
  int fin_found;
  // broadcasts
  uint32_t b_prefix;
  unsigned long long b_mass;
  uint32_t b_ties;
  uint32_t b_ties_before;  // entries equal to the threshold in lower-ranked CTAs
  uint32_t b_ties_mine;    // and in this CTA
  unsigned long long b_u;
  float b_f;
  int b_i;
  float thr;
  int found;
};

__host__ __device__ constexpr size_t n16_list_offset(int per_cta) {
  return (static_cast<size_t>(per_cta) * 2 + 15) / 16 * 16;
}
__host__ __device__ constexpr size_t n16_smem_bytes(int per_cta) {
  return n16_list_offset(per_cta) + static_cast<size_t>(kN16ListCap) * (sizeof(N16Idx) + 4);
}

template <typename In>
__device__ __forceinline__ float h16_to_f32(uint16_t b) {
  return to_f32<In>(*reinterpret_cast<const In*>(&b));
}

// x / d rounded to nearest even by Markstein's correction of x * RN(1/d) (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990): with r = RN(1/d) and q0 = RN(x r), the fused q0 + r * (x - d q0) rounds
// to RN(x / d) whenever nothing leaves the normal range -- guaranteed here by |x| and d in
// [2^-60, 2^60] and [2^-30, 2^30]; other arguments take the IEEE division.  Three
// instructions instead of the division's sequence.
__device__ __forceinline__ float div_rn(float x, float d, float r, bool d_ok) {
  const float ax = fabsf(x);
  if (d_ok && ax >= 0x1p-60f && ax <= 0x1p60f) {
    const float q0 = __fmul_rn(x, r);
    return __fmaf_rn(__fmaf_rn(-q0, d, x), r, q0);
  }
  return __fdiv_rn(x, d);
}
__device__ __forceinline__ bool div_ok(float d) { return d >= 0x1p-30f && d <= 0x1p30f; }

// p(x) = RN(expf(RN(x / T) - ymax) / z), the probability sampling_kernel computes
struct N16Prob {
  float temp, rt, ymax, z, rz;
  bool t_ok, z_ok;
  __device__ __forceinline__ float y(float x) const { return div_rn(x, temp, rt, t_ok); }
  __device__ __forceinline__ float e(float x) const { return expf(y(x) - ymax); }
  __device__ __forceinline__ float operator()(float x) const { return div_rn(e(x), z, rz, z_ok); }
};

// The radix select of sampling_kernel over an entry set given by `each(f)`, which calls
// f(p) for every entry of this CTA: four 8-bit passes over the bits of p, masses in units of
// 2^-31, histograms combined across the cluster in rank order.  Returns the threshold bits
// and sets `above` (the mass of entries above them) and `ties` (entries equal to them).
// Per pass: the histogram, one block barrier, the cluster barrier, then warp 0 alone reads
// the cluster's bins (16-byte loads of its 8 bins from every CTA) and picks the digit while
// the other warps clear the histogram buffer the pass after next will use (every CTA has
// read it once this pass's cluster barrier is passed), and one more block barrier.
template <int C, bool kCluster, class Each>
__device__ uint32_t n16_radix_select(N16Shared& sh, unsigned long long limit, Each each,
                                     unsigned long long& above_out, uint32_t& ties_out,
                                     uint32_t& ties_before_out, uint32_t& ties_mine_out,
                                     int shift_hi = 24, int shift_lo = 0, uint32_t prefix_in = 0,
                                     unsigned long long above_in = 0) {
  constexpr int R = kCluster ? C : 1;  // CTAs whose histograms are summed
  const int tid = threadIdx.x, lane = tid & 31;
  if (shift_hi == 24) {
    // a continuation (shift_hi < 24) finds its buffer cleared by the previous pass
    for (int b = tid; b < 2 * 256; b += kN16Threads) {
      (&sh.hist_m[0][0])[b] = 0;
      (&sh.hist_c[0][0])[b] = 0;
    }
    __syncthreads();
  }
  uint32_t prefix = prefix_in;
  unsigned long long above = above_in;
  uint32_t ties = 0;
  for (int shift = shift_hi; shift >= shift_lo; shift -= 8) {
    const int buf = (shift >> 3) & 1;
    uint32_t* hm = sh.hist_m[buf];
    uint32_t* hc = sh.hist_c[buf];
    const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
    each([&](float v) {
      const uint32_t bits = __float_as_uint(v);
      if ((bits & hi_mask) == (prefix & hi_mask)) {
        const uint32_t d = (bits >> shift) & 255u;
        atomicAdd(&hm[d], to_q31(v));
        atomicAdd(&hc[d], 1u);
      }
    });
    __syncthreads();
    if (kCluster) samp_cluster_sync();  // every CTA's histogram is complete; the other buffer is free
    if (tid < 32) {
      // lane l owns bins 255 - 8l .. 248 - 8l (descending); the cut bin is the lowest
      // non-empty bin whose mass above (above + all higher bins) is within the limit
      const int b0 = 248 - 8 * lane;
      unsigned long long m8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      uint32_t c8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      uint4 vm[R][2], vc[R][2];  // every CTA's bins first, so the loads are in flight together
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint4* pm = kCluster ? cl_ptr(reinterpret_cast<const uint4*>(hm + b0), static_cast<uint32_t>(r))
                                   : reinterpret_cast<const uint4*>(hm + b0);
        const uint4* pc = kCluster ? cl_ptr(reinterpret_cast<const uint4*>(hc + b0), static_cast<uint32_t>(r))
                                   : reinterpret_cast<const uint4*>(hc + b0);
        vm[r][0] = pm[0];
        vm[r][1] = pm[1];
        vc[r][0] = pc[0];
        vc[r][1] = pc[1];
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint4 ma = vm[r][0], mb = vm[r][1], ca = vc[r][0], cb = vc[r][1];
        m8[0] += ma.x; m8[1] += ma.y; m8[2] += ma.z; m8[3] += ma.w;
        m8[4] += mb.x; m8[5] += mb.y; m8[6] += mb.z; m8[7] += mb.w;
        c8[0] += ca.x; c8[1] += ca.y; c8[2] += ca.z; c8[3] += ca.w;
        c8[4] += cb.x; c8[5] += cb.y; c8[6] += cb.z; c8[7] += cb.w;
      }
      unsigned long long mine = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) mine += m8[j];
      unsigned long long pre = mine;  // inclusive scan in lane order (descending bins)
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long t = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += t;
      }
      unsigned long long acc = above + pre - mine;
      int cand = 256;
      unsigned long long cand_acc = 0;
      uint32_t cand_cnt = 0;
#pragma unroll
      for (int j = 7; j >= 0; --j) {  // bins b0 + 7 .. b0, descending
        if (c8[j] > 0 && acc <= limit) {
          cand = b0 + j;
          cand_acc = acc;
          cand_cnt = c8[j];
        }
        acc += m8[j];
      }
      int best = cand;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = min(best, __shfl_xor_sync(0xffffffffu, best, o));
      if (best == 256) best = 0;  // not reached: the largest entry always qualifies
      const uint32_t owner = static_cast<uint32_t>((255 - best) / 8);
      const unsigned long long best_acc = __shfl_sync(0xffffffffu, cand_acc, owner);
      const uint32_t best_cnt = __shfl_sync(0xffffffffu, cand_cnt, owner);
      if (lane == 0) {
        sh.b_prefix = prefix | (static_cast<uint32_t>(best) << shift);
        sh.b_mass = best_acc;
        sh.b_ties = best_cnt;
      }
      if (shift == 0) {
        // the final bin holds exactly the entries equal to the threshold: its count in each
        // CTA (lane r reads CTA r's), split into the CTAs ranked below this one and this CTA
        const uint32_t me = kCluster ? samp_rank() : 0u;
        uint32_t cnt = 0;
        if (lane < R) cnt = kCluster ? *cl_ptr(hc + best, static_cast<uint32_t>(lane)) : hc[best];
        uint32_t before = static_cast<uint32_t>(lane) < me ? cnt : 0u;
        uint32_t mine = static_cast<uint32_t>(lane) == me ? cnt : 0u;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          before += __shfl_xor_sync(0xffffffffu, before, o);
          mine += __shfl_xor_sync(0xffffffffu, mine, o);
        }
        if (lane == 0) {
          sh.b_ties_before = before;
          sh.b_ties_mine = mine;
        }
      }
    } else if (shift > 0) {
      uint32_t* zm = sh.hist_m[buf ^ 1];
      uint32_t* zc = sh.hist_c[buf ^ 1];
      for (int b = tid - 32; b < 256; b += kN16Threads - 32) {
        zm[b] = 0;
        zc[b] = 0;
      }
    }
    __syncthreads();
    prefix = sh.b_prefix;
    above = sh.b_mass;
    ties = sh.b_ties;
  }
  const uint32_t tb = sh.b_ties_before, tm = sh.b_ties_mine;
  __syncthreads();  // the broadcast slots are reused by the caller
  above_out = above;
  ties_out = ties;
  ties_before_out = tb;
  ties_mine_out = tm;
  return prefix;
}

// Index of the k-th (0-based) entry, in index order, for which pred(i) holds among the
// `count` entries i = 0 .. count-1 of this CTA; -1 if there are not that many.  Entries are
// taken in chunks of 8 consecutive per thread.  Block-uniform call.
template <class Pred>
__device__ int n16_kth(N16Shared& sh, int count, unsigned long long k, Pred pred) {
  const int tid = threadIdx.x;
  if (tid == 0) sh.found = -1;
  __syncthreads();
  unsigned long long acc = 0;
  for (int c0 = 0; c0 < count; c0 += kN16Chunk) {
    const int i0 = c0 + tid * 8;
    uint32_t bits = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (i0 + j < count && pred(i0 + j)) bits |= 1u << j;
    unsigned long long tot;
    const unsigned long long ex = acc + block_exscan_u64(sh, __popc(bits), tot);
    if (k >= ex && k < ex + __popc(bits)) {
      unsigned long long r = ex;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (bits & (1u << j)) {
          if (r == k) sh.found = i0 + j;
          ++r;
        }
    }
    acc += tot;
    __syncthreads();
    if (sh.found >= 0) break;
  }
  const int f = sh.found;
  __syncthreads();
  return f;
}

// mode 0 only, In = bf16 or f16.
template <int C, typename In>
__global__ void __launch_bounds__(kN16Threads, kN16CtasPerSm) nucleus16_kernel(const SampParams p) {
  extern __shared__ __align__(16) uint8_t n16_dyn[];
  __shared__ N16Shared sh;
  uint16_t* xs = reinterpret_cast<uint16_t*>(n16_dyn);
  N16Idx* lidx = reinterpret_cast<N16Idx*>(n16_dyn + n16_list_offset(p.per_cta));
  float* lp = reinterpret_cast<float*>(n16_dyn + n16_list_offset(p.per_cta) + kN16ListCap * sizeof(N16Idx));
  const int tid = threadIdx.x;
  const uint32_t rank = samp_rank();
  const int row = blockIdx.x / C;
  const int64_t lo = static_cast<int64_t>(rank) * p.per_cta;
  int n = static_cast<int>(p.vocab - lo < p.per_cta ? p.vocab - lo : p.per_cta);
  if (n < 0) n = 0;
  const uint16_t* src = static_cast<const uint16_t*>(p.src) + static_cast<int64_t>(row) * p.stride + lo;
  const float temp = p.temps ? p.temps[row] : p.temp;
  const float top_p = p.top_ps ? p.top_ps[row] : p.top_p;
  const bool greedy = !(temp > 0.f);
  grid_dependency_wait();  // launched early behind the previous kernel on the stream

  // ---- phase 1: stage the raw logits; per thread the running max of x and the sum z of
  // 2^(x log2(e)/T - y(max) log2 e) relative to it (rescaled when the max grows), so one
  // pass and one cluster exchange give the row max and z.  A term costs one fma and one
  // ex2: it differs from expf(x/T - y(max)) by a few parts in 10^6 at most, and z is a sum
  // of such terms (the probabilities themselves are computed exactly below).
  N16Prob pr;
  pr.temp = temp;
  pr.rt = greedy ? 0.f : __frcp_rn(temp);
  pr.t_ok = !greedy && div_ok(temp);
  constexpr float kLog2e = 1.4426950408889634f;
  const float c1 = greedy ? 0.f : kLog2e * pr.rt;  // log2(e) / T
  float mx = -INFINITY, zs = 0.f;
  // fold cnt values whose max is cm into (mx, zs)
  auto absorb = [&](const float* f, int cnt, float cm) {
    if (greedy) {
      mx = fmaxf(mx, cm);
      return;
    }
    if (cm > mx) {
      if (zs != 0.f) zs *= ex2(__fmul_rn(pr.y(mx) - pr.y(cm), kLog2e));
      mx = cm;
    }
    if (mx == -INFINITY) return;
    const float c2 = pr.y(mx) * kLog2e;
    for (int j = 0; j < cnt; ++j) zs += ex2(fmaf(f[j], c1, -c2));
  };
  {
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const int nv = n / 8;
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
      uint4* x4 = reinterpret_cast<uint4*>(xs);
#pragma unroll 2
      for (int v = tid; v < nv; v += kN16Threads) {
        const uint4 raw = __ldg(s4 + v);
        x4[v] = raw;
        const uint16_t* h = reinterpret_cast<const uint16_t*>(&raw);
        float f[8];
        float cm = -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          f[j] = h16_to_f32<In>(h[j]);
          cm = fmaxf(cm, f[j]);
        }
        absorb(f, 8, cm);
      }
      done = nv * 8;
    }
    for (int i = done + tid; i < n; i += kN16Threads) {
      const uint16_t b = src[i];
      xs[i] = b;
      const float f = h16_to_f32<In>(b);
      absorb(&f, 1, f);
    }
  }
  float bmax = mx;
  {
    int dummy = 0;
    block_argmax(sh, bmax, dummy);
  }
  float bz = 0.f;
  if (!greedy && zs != 0.f) bz = zs * ex2(__fmul_rn(pr.y(mx) - pr.y(bmax), kLog2e));
  bz = block_sum_f32(sh, bz);
  if (tid == 0) {
    sh.x_mz[0] = bmax;
    sh.x_mz[1] = bz;
  }
  grid_launch_dependents();  // the next call's CTAs may launch as this one's retire
  samp_cluster_sync();
  float xmax = -INFINITY;
#pragma unroll
  for (int r = 0; r < C; ++r) xmax = fmaxf(xmax, ld_cl_f32(&sh.x_mz[0], r));

  float* out = p.probs_out ? p.probs_out + static_cast<int64_t>(row) * p.out_stride + lo : nullptr;
  if (greedy) {
    // T <= 0: one-hot at the first index holding the max (core/spec_decode.py:18-21)
    int first = 0x7fffffff;
    for (int i = tid; i < n; i += kN16Threads)
      if (h16_to_f32<In>(xs[i]) == xmax && static_cast<int>(lo) + i < first) first = static_cast<int>(lo) + i;
    float fv = 0.f;  // equal values: block_argmax keeps the smallest index
    block_argmax(sh, fv, first);
    if (tid == 0) sh.x_i = first;
    samp_cluster_sync();
    int gidx = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < C; ++r) gidx = min(gidx, static_cast<int>(ld_cl_u32(&sh.x_i, r)));
    samp_cluster_sync();
    if (out)
      for (int i = tid; i < n; i += kN16Threads) out[i] = (static_cast<int>(lo) + i == gidx) ? 1.f : 0.f;
    if (p.tokens && rank == 0 && tid == 0) p.tokens[row] = gidx;
    return;
  }

  // ---- phase 2: z = sum of exp(x / T - ymax), the CTAs' sums moved to the row max
  pr.ymax = __fdiv_rn(xmax, temp);
  float z = 0.f;
  {
    float cm[C], cz[C];  // every CTA's (max, z) loaded first, so the remote loads overlap
#pragma unroll
    for (int r = 0; r < C; ++r) {
      cm[r] = ld_cl_f32(&sh.x_mz[0], r);
      cz[r] = ld_cl_f32(&sh.x_mz[1], r);
    }
#pragma unroll
    for (int r = 0; r < C; ++r)
      if (cz[r] != 0.f) z += cz[r] * ex2(__fmul_rn(pr.y(cm[r]) - pr.ymax, kLog2e));
  }
  pr.z = z;
  pr.rz = __frcp_rn(z);
  pr.z_ok = div_ok(z);
  auto prob = [&](int i) { return pr(h16_to_f32<In>(xs[i])); };

  // ---- phase 3: candidates (only with a cut)
  const bool cut = top_p < 1.f;
  const unsigned long long limit = __double2ull_rn(static_cast<double>(top_p) * 2147483648.0);
  bool fast = false;
  int count = 0;
  if (cut) {
    if (tid == 0) {
      const double v = static_cast<double>(p.vocab);
      const double qmin = (2147483648.0 * (1.0 - 1.0 / 4096.0) - 0.5 * v - static_cast<double>(limit)) / v - 1.0;
      float thr = -INFINITY;
      if (qmin > 0.0) {
        // p >= p_min needs x / T >= ymax + ln(p_min z) up to the rounding of the division,
        // expf, the subtraction and logf (relative 2^-20 or less); the margin is orders of
        // magnitude wider
        const float lq = logf(__double2float_rd(qmin / 2147483648.0));
        float t = pr.ymax + lq + logf(z);
        t -= 1e-3f + 1e-5f * fabsf(t);
        const float xt = t * temp;
        thr = xt - 1e-5f * fabsf(xt);
      }
      sh.thr = thr;
    }
    __syncthreads();
    const float thr = sh.thr;
    // The candidate indices in index order, in one pass: warp w owns the contiguous
    // entries [w * per_w, (w + 1) * per_w) and list slots [w * kWarpCap, (w + 1) * kWarpCap);
    // lanes take 8 consecutive entries per 256-entry chunk, a warp scan places them.  Slots
    // past a warp's candidates hold p = 0, which every later step skips (no mass, below any
    // threshold), so the list is read as kN16ListCap slots in index order.
    constexpr int kWarpCap = kN16ListCap / kSampWarps;
    const int warp = tid >> 5, lane = tid & 31;
    const int per_w = ((n + kSampWarps - 1) / kSampWarps + 7) / 8 * 8;
    const int w0 = min(n, warp * per_w), w1 = min(n, w0 + per_w);
    auto lane_bits = [&](int i0) -> uint32_t {
      uint32_t bits = 0;
      if (i0 + 8 <= w1) {
        const uint4 raw = reinterpret_cast<const uint4*>(xs)[i0 / 8];
        const uint16_t* h = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (h16_to_f32<In>(h[j]) >= thr) bits |= 1u << j;
      } else {
        for (int j = 0; j < 8; ++j)
          if (i0 + j < w1 && h16_to_f32<In>(xs[i0 + j]) >= thr) bits |= 1u << j;
      }
      return bits;
    };
    N16Idx* wl = lidx + warp * kWarpCap;
    int wc = 0;  // this warp's candidates so far
#pragma unroll 2
    for (int c = w0; c < w1; c += 256) {
      uint32_t bits = lane_bits(c + 8 * lane);
      const int mine = __popc(bits);
      int incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
      }
      int at = wc + incl - mine;
      while (bits) {
        const int j = __ffs(bits) - 1;
        bits &= bits - 1;
        if (at < kWarpCap) wl[at] = static_cast<N16Idx>(c + 8 * lane + j);
        ++at;
      }
      wc += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) sh.wi[warp] = wc;
    __syncthreads();
    bool over = false;
    for (int w = 0; w < kSampWarps; ++w) over |= sh.wi[w] > kWarpCap;
    for (int j = tid; j < kN16ListCap; j += kN16Threads) {
      const int w = j / kWarpCap;
      lp[j] = j - w * kWarpCap < sh.wi[w] ? prob(lidx[j]) : 0.f;
    }
    __syncthreads();
    // A CTA whose list overflowed takes the full path alone: every entry off the list has
    // p below the proven bound, under the threshold, so it adds only to histogram bins
    // below each pass's cut bin and never to the kept set.
    fast = !over;
    count = kN16ListCap;
  }
  // every entry of this CTA's set, as f(p) (list entries, or every logit)
  auto each = [&](auto&& f) {
    if (fast) {
      for (int j = tid; j < count; j += kN16Threads) f(lp[j]);
    } else {
      for (int i = tid; i < n; i += kN16Threads) f(prob(i));
    }
  };

  // ---- phase 4: top-p threshold, then the index at which a tied group is cut
  constexpr float kFx = 4503599627370496.0f;
  uint32_t tbits = 0;
  int i_cut = 0x7fffffff;  // ties at tbits are kept below this global index
  bool finished = false;
  unsigned long long above = 0;
  uint32_t ties = 0, ties_before = 0, ties_mine = 0;
  if (cut) {
    // two 8-bit passes locate the threshold's 16-bit prefix (exponent and 7 mantissa bits)
    const uint32_t pre = n16_radix_select<C, true>(sh, limit, each, above, ties, ties_before, ties_mine, 24, 16);
    if (ties <= static_cast<uint32_t>(kN16Fin)) {
      // Few entries share it (bf16 logits make them largely exact ties): every CTA lists its
      // own, and warp 0 of each CTA orders all of them by (p desc, index asc) and walks
      // their masses from `above`.  The first entry whose exclusive mass exceeds the limit
      // is the first one dropped: the kept set is everything before it in that order.
      if (tid == 0) sh.fin_n = 0;
      __syncthreads();
      auto take = [&](float v, int gi) {
        const uint32_t b = __float_as_uint(v);
        if ((b >> 16) == (pre >> 16)) {
          const int at = atomicAdd(&sh.fin_n, 1);
          if (at < kN16Fin) {
            sh.fin_bits[at] = b;
            sh.fin_idx[at] = gi;
          }
        }
      };
      if (fast) {
        for (int j = tid; j < count; j += kN16Threads) take(lp[j], static_cast<int>(lo) + lidx[j]);
      } else {
        for (int i = tid; i < n; i += kN16Threads) take(prob(i), static_cast<int>(lo) + i);
      }
      __syncthreads();
      samp_cluster_sync();  // every CTA's list is complete
      if (tid < 32) {
        const int lane = tid;
        // entries e = lane and lane + 32 of the cluster's lists in rank order
        unsigned long long key[2] = {~0ull, ~0ull};
        int tot = 0;
#pragma unroll
        for (int r = 0; r < C; ++r) {
          const int nr = min(static_cast<int>(ld_cl_u32(&sh.fin_n, r)), kN16Fin);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int e = lane + 32 * h - tot;
            if (e >= 0 && e < nr) {
              const uint32_t b = *cl_ptr(sh.fin_bits + e, r);
              const int gi = *cl_ptr(sh.fin_idx + e, r);
              key[h] = (static_cast<unsigned long long>(~b) << 32) | static_cast<uint32_t>(gi);
            }
          }
          tot += nr;
        }
        // rank of each entry among the (at most 64) keys, then the keys in order (unused
        // slots keep the largest key)
        sh.fin_key[lane] = ~0ull;
        sh.fin_key[lane + 32] = ~0ull;
        __syncwarp();
        int rank[2] = {0, 0};
        for (int src = 0; src < 64; ++src) {
          const unsigned long long k = __shfl_sync(0xffffffffu, key[src >> 5], src & 31);
#pragma unroll
          for (int h = 0; h < 2; ++h) rank[h] += k < key[h] ? 1 : 0;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (key[h] != ~0ull) sh.fin_key[rank[h]] = key[h];  // distinct: the index is in the key
        __syncwarp();
        // exclusive masses in order: lane holds positions 2 lane, 2 lane + 1
        const unsigned long long k0 = sh.fin_key[2 * lane], k1 = sh.fin_key[2 * lane + 1];
        const uint32_t m0 = k0 == ~0ull ? 0u : to_q31(__uint_as_float(~static_cast<uint32_t>(k0 >> 32)));
        const uint32_t m1 = k1 == ~0ull ? 0u : to_q31(__uint_as_float(~static_cast<uint32_t>(k1 >> 32)));
        unsigned long long incl = static_cast<unsigned long long>(m0) + m1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const unsigned long long t = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += t;
        }
        const unsigned long long ex0 = above + incl - m0 - m1, ex1 = ex0 + m0;
        int first = 64;
        if (k1 != ~0ull && ex1 > limit) first = 2 * lane + 1;
        if (k0 != ~0ull && ex0 > limit) first = 2 * lane;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
        if (lane == 0) {
          sh.fin_found = first < tot ? 1 : 0;
          if (first < tot) {
            const unsigned long long kc = sh.fin_key[first];
            sh.fin_cut_bits = ~static_cast<uint32_t>(kc >> 32);
            sh.fin_cut_idx = static_cast<int>(static_cast<uint32_t>(kc));
          }
        }
      }
      __syncthreads();
      if (sh.fin_found) {
        tbits = sh.fin_cut_bits;
        i_cut = sh.fin_cut_idx;
        finished = true;
      }
    }
    if (!finished) {
      // the last two passes, from the 16-bit prefix
      tbits = n16_radix_select<C, true>(sh, limit, each, above, ties, ties_before, ties_mine, 8, 0, pre, above);
    }
  }
  if (cut && !finished) {
    const unsigned long long tq = to_q31(__uint_as_float(tbits));
    uint32_t keep_ties = ties;
    if (tq > 0) {
      const unsigned long long room = (limit - above) / tq + 1;  // above <= limit
      if (room < keep_ties) keep_ties = static_cast<uint32_t>(room);
    }
    if (keep_ties < ties) {
      // the ties are kept in index order: the first keep_ties of them, of which this CTA
      // (after ties_before in lower-ranked CTAs) keeps its first keep_mine
      const uint32_t keep_mine =
          keep_ties <= ties_before ? 0u : min(ties_mine, keep_ties - ties_before);
      if (keep_mine == 0) {
        i_cut = static_cast<int>(lo);  // none of this CTA's ties
      } else if (keep_mine < ties_mine) {
        int local_cut = fast ? n16_kth(sh, count, keep_mine, [&](int j) { return __float_as_uint(lp[j]) == tbits; })
                             : n16_kth(sh, n, keep_mine, [&](int i) { return __float_as_uint(prob(i)) == tbits; });
        if (fast && local_cut >= 0) local_cut = lidx[local_cut];
        if (local_cut >= 0) i_cut = static_cast<int>(lo) + local_cut;
      }
    }
  }
  auto kept = [&](float v, int gi) {
    const uint32_t b = __float_as_uint(v);
    return !cut || b > tbits || (b == tbits && gi < i_cut);
  };

  // ---- kept mass in units of 2^-52: this CTA's share, the shares before it, the total
  unsigned long long local = 0;
  if (fast) {
    for (int j = tid; j < count; j += kN16Threads) {
      const float v = lp[j];
      if (kept(v, static_cast<int>(lo) + lidx[j])) local += to_fixed(v, kFx);
    }
  } else {
    for (int i = tid; i < n; i += kN16Threads) {
      const float v = prob(i);
      if (kept(v, static_cast<int>(lo) + i)) local += to_fixed(v, kFx);
    }
  }
  local = block_sum_u64(sh, local);
  if (tid == 0) sh.x_kept = local;
  // split cluster barrier: the zero fill of the output (which needs no total) runs between
  // this CTA's arrival and its wait for the others'
  samp_cluster_arrive();
  if (out && fast) {
    int done = 0;
    if ((reinterpret_cast<uintptr_t>(out) & 15) == 0) {
      const int nv = n / 4;
      float4* out4 = reinterpret_cast<float4*>(out);
      for (int v = tid; v < nv; v += kN16Threads) out4[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      done = nv * 4;
    }
    for (int i = done + tid; i < n; i += kN16Threads) out[i] = 0.f;
  }
  __syncthreads();  // every zero store of this CTA's slice before any scatter into it
  samp_cluster_wait();
  unsigned long long base = 0, total = 0;
#pragma unroll
  for (int r = 0; r < C; ++r) {
    const unsigned long long v = ld_cl_u64(&sh.x_kept, r);
    if (r < static_cast<int>(rank)) base += v;
    total += v;
  }

  // ---- phase 5: renormalised probabilities
  if (out) {
    const float s = static_cast<float>(static_cast<double>(total) / kFixedOne);
    if (fast) {
      // zeros everywhere (above), then the kept candidates
      for (int j = tid; j < count; j += kN16Threads) {
        const float v = lp[j];
        if (v > 0.f && kept(v, static_cast<int>(lo) + lidx[j])) out[lidx[j]] = __fdiv_rn(v, s);
      }
    } else {
      for (int i = tid; i < n; i += kN16Threads) {
        const float v = prob(i);
        out[i] = (v > 0.f && kept(v, static_cast<int>(lo) + i)) ? __fdiv_rn(v, s) : 0.f;
      }
    }
  }

  // ---- phase 6: one draw, inverse CDF in index order over the kept masses
  if (p.tokens && total == 0) {
    if (rank == 0 && tid == 0) {
      p.tokens[row] = -1;
      report_error(p.error_word, INFERD_ERR_INVALID_ARGUMENT);
    }
  } else if (p.tokens) {
    const unsigned long long target = __umul64hi(philox_u64(p.seed, p.offset + static_cast<uint64_t>(row)), total);
    if (target >= base && target < base + local) {
      // weights of the entries of this CTA in index order (candidates or every logit)
      const int m = fast ? count : n;
      if (tid == 0) sh.found = 0;
      __syncthreads();
      unsigned long long acc0 = base;
      for (int c0 = 0; c0 < m; c0 += kN16Chunk) {
        const int i0 = c0 + tid * 8;
        unsigned long long q[8];
        unsigned long long mine = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          q[j] = 0;
          if (i0 + j < m) {
            const int li = fast ? lidx[i0 + j] : i0 + j;
            const float v = fast ? lp[i0 + j] : prob(i0 + j);
            if (kept(v, static_cast<int>(lo) + li)) q[j] = to_fixed(v, kFx);
          }
          mine += q[j];
        }
        unsigned long long tot_chunk;
        const unsigned long long ex = acc0 + block_exscan_u64(sh, mine, tot_chunk);
        if (target >= ex && target < ex + mine) {
          unsigned long long acc = ex;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc += q[j];
            if (acc > target) {
              p.tokens[row] = lo + (fast ? lidx[i0 + j] : i0 + j);
              sh.found = 1;
              break;
            }
          }
        }
        acc0 += tot_chunk;
        __syncthreads();
        if (sh.found) break;
      }
    }
  }
  // no CTA leaves while another may still read its exchange slots
  samp_cluster_sync();
}

template <int C, typename In>
int launch_nucleus16(const SampParams& p, cudaStream_t s) {
  const size_t smem = n16_smem_bytes(p.per_cta);
  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(nucleus16_kernel<C, In>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(n16_smem_bytes(kN16MaxPerCta)));
    if (e != cudaSuccess) return cuda_status(e);
    e = cudaFuncSetAttribute(nucleus16_kernel<C, In>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows) * C);
  cfg.blockDim = dim3(kN16Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cuda_status(cudaLaunchKernelEx(&cfg, nucleus16_kernel<C, In>, p));
}

// 16-bit logits: the candidate kernel when a row fits 8 CTAs' shared memory; false otherwise
template <typename In>
bool dispatch_nucleus16(SampParams& p, cudaStream_t s, int* status) {
  int c = 1;
  while (c < 8 && (p.vocab + c - 1) / c > kN16MaxPerCta) c <<= 1;
  const int64_t per = ((p.vocab + c - 1) / c + 7) / 8 * 8;  // 16-byte aligned CTA slices
  if (per > kN16MaxPerCta) return false;
  p.per_cta = static_cast<int32_t>(per);
  switch (c) {
    case 1: *status = launch_nucleus16<1, In>(p, s); break;
    case 2: *status = launch_nucleus16<2, In>(p, s); break;
    case 4: *status = launch_nucleus16<4, In>(p, s); break;
    default: *status = launch_nucleus16<8, In>(p, s); break;
  }
  return true;
}

// ---------------------------------------------------------------- speculative accept / resample
// core/spec_decode.py:145-161 for a batch of sequences in one launch.  For sequence b, draft
// token k (x = proposals[b][k]) is accepted when u_k <= p[b][k][x] / q[b][k][x] (fp32
// division; u_k uniform on the float32 grid of [0, 1), Philox stream 1 + k).  At the first
// rejection one token is drawn from clamp(p[b][k] - q[b][k], 0) -- from p[b][k] when that is
// all zero -- and the round ends; when all gamma drafts are accepted the bonus token is drawn
// from p[b][gamma].  The draw is sample_from's rule (power-of-two fixed point, inverse CDF in
// index order, Philox stream 0), so the reference's loop of host syncs (one .item() per draft
// token) becomes one launch.  One cluster of C CTAs per sequence; CTA r scans entries
// [r * per_cta, (r + 1) * per_cta) of the chosen distribution straight from global memory.
constexpr int kSpecThreads = 512;

struct SpecParams {
  const float* p;            // [rows][gamma + 1][vocab] at strides p_row, p_dist
  const float* q;            // [rows][gamma][vocab]     at strides q_row, q_dist
  int64_t p_row, p_dist, q_row, q_dist;
  const int64_t* proposals;  // [rows][prop_row]
  int64_t prop_row;
  int32_t rows, gamma;
  int64_t vocab;
  int32_t per_cta;
  int32_t* accepted;         // [rows]
  int64_t* tokens;           // [rows][tok_row], gamma + 1 used: accepted drafts, the draw, -1
  int64_t tok_row;
  uint64_t seed, offset;
  int32_t* error_word;
};

struct SpecShared {
  float wf[kSampWarps];
  int wi[kSampWarps];
  unsigned long long wu[kSampWarps];
  float b_f;
  int b_i;
  unsigned long long b_u;
  float x_f;
  unsigned long long x_u;
  int kstar;
  int found;
};

__device__ __forceinline__ float spec_uniform(uint64_t seed, uint64_t n, uint32_t stream) {
  uint32_t c[4] = {static_cast<uint32_t>(n), static_cast<uint32_t>(n >> 32), stream, 0u};
  uint32_t k0 = static_cast<uint32_t>(seed), k1 = static_cast<uint32_t>(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    philox_round(c, k0, k1);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return static_cast<float>(c[0] >> 8) * 0x1p-24f;
}

template <int C>
__global__ void __launch_bounds__(kSpecThreads) spec_accept_kernel(const SpecParams p) {
  __shared__ SpecShared sh;
  const int tid = threadIdx.x;
  const uint32_t rank = samp_rank();
  const int row = blockIdx.x / C;
  const int64_t lo = static_cast<int64_t>(rank) * p.per_cta;
  int n = static_cast<int>(p.vocab - lo < p.per_cta ? p.vocab - lo : p.per_cta);
  if (n < 0) n = 0;
  const uint64_t ctr = p.offset + static_cast<uint64_t>(row);
  const float* prow = p.p + static_cast<int64_t>(row) * p.p_row;
  const float* qrow = p.q + static_cast<int64_t>(row) * p.q_row;
  const int64_t* props = p.proposals + static_cast<int64_t>(row) * p.prop_row;

  // ---- the accept decisions (cheap: gamma ratios), the same in every CTA of the cluster
  if (tid == 0) {
    int kstar = p.gamma;
    for (int k = 0; k < p.gamma; ++k) {
      const int64_t x = props[k];
      if (x < 0 || x >= p.vocab) {  // not a token: rejected (and reported)
        report_error(p.error_word, INFERD_ERR_INVALID_ARGUMENT);
        kstar = k;
        break;
      }
      const float ratio = __fdiv_rn(prow[k * p.p_dist + x], qrow[k * p.q_dist + x]);
      if (!(spec_uniform(p.seed, ctr, 1u + static_cast<uint32_t>(k)) <= ratio)) {
        kstar = k;
        break;
      }
    }
    sh.kstar = kstar;
  }
  __syncthreads();
  const int kstar = sh.kstar;
  const bool resid = kstar < p.gamma;
  const float* pd = prow + static_cast<int64_t>(kstar) * p.p_dist + lo;
  const float* qd = resid ? qrow + static_cast<int64_t>(kstar) * p.q_dist + lo : nullptr;

  // ---- weights: the residual clamp(p - q, 0), else the bonus distribution; a residual with
  // no positive entry falls back to p (the reference's `total > 0` test)
  bool use_q = resid;
  float fxs = 0.f;
  unsigned long long local = 0, base = 0, total = 0;
  for (int attempt = 0; attempt < 2; ++attempt) {
    auto weight = [&](int i) {
      const float a = __ldg(pd + i);
      return use_q ? fmaxf(a - __ldg(qd + i), 0.f) : a;
    };
    float wmax = 0.f;
    bool bad = false;
    for (int i = tid; i < n; i += kSpecThreads) {
      const float w = weight(i);
      if (!(w >= 0.f) || w == INFINITY) bad = true;
      else wmax = fmaxf(wmax, w);
    }
    if (bad) report_error(p.error_word, INFERD_ERR_INVALID_ARGUMENT);
    int dummy = 0;
    block_argmax(sh, wmax, dummy);
    if (tid == 0) sh.x_f = wmax;
    samp_cluster_sync();
    float gmax = 0.f;
#pragma unroll
    for (int r = 0; r < C; ++r) gmax = fmaxf(gmax, ld_cl_f32(&sh.x_f, r));
    samp_cluster_sync();
    // 2^(52 - k) with 2^k >= vocab * max weight (sample_from's scale)
    int ex = 0;
    frexpf(gmax, &ex);
    const int lv = p.vocab > 1 ? 64 - __clzll(static_cast<unsigned long long>(p.vocab - 1)) : 0;
    int kk = ex + lv;
    if (kk < 0) kk = 0;
    fxs = ldexpf(1.f, 52 - kk);
    local = 0;
    for (int i = tid; i < n; i += kSpecThreads) {
      const float w = weight(i);
      if (w >= 0.f && w != INFINITY) local += to_fixed(w, fxs);
    }
    local = block_sum_u64(sh, local);
    if (tid == 0) sh.x_u = local;
    samp_cluster_sync();
    base = 0;
    total = 0;
#pragma unroll
    for (int r = 0; r < C; ++r) {
      const unsigned long long v = ld_cl_u64(&sh.x_u, r);
      if (r < static_cast<int>(rank)) base += v;
      total += v;
    }
    samp_cluster_sync();
    if (total > 0 || !use_q) break;
    use_q = false;  // all-zero residual: draw from p[kstar] itself
  }

  // ---- outputs: the accepted drafts and the count (CTA 0), then the draw
  int64_t* tok = p.tokens + static_cast<int64_t>(row) * p.tok_row;
  if (rank == 0) {
    for (int k = tid; k <= p.gamma; k += kSpecThreads) {
      if (k < kstar) tok[k] = props[k];
      else if (k > kstar) tok[k] = -1;
    }
    if (tid == 0) p.accepted[row] = kstar;
  }
  if (total == 0) {
    if (rank == 0 && tid == 0) {
      tok[kstar] = -1;
      report_error(p.error_word, INFERD_ERR_INVALID_ARGUMENT);
    }
    return;
  }
  const unsigned long long target = __umul64hi(philox_u64(p.seed, ctr), total);
  if (target >= base && target < base + local) {
    if (tid == 0) sh.found = 0;
    __syncthreads();
    unsigned long long acc0 = base;
    for (int c0 = 0; c0 < n; c0 += kSpecThreads * 8) {
      const int i0 = c0 + tid * 8;
      unsigned long long qv[8];
      unsigned long long mine = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        qv[j] = 0;
        if (i0 + j < n) {
          const float a = __ldg(pd + i0 + j);
          const float w = use_q ? fmaxf(a - __ldg(qd + i0 + j), 0.f) : a;
          if (w >= 0.f && w != INFINITY) qv[j] = to_fixed(w, fxs);
        }
        mine += qv[j];
      }
      unsigned long long tot_chunk;
      const unsigned long long ex = acc0 + block_exscan_u64(sh, mine, tot_chunk);
      if (target >= ex && target < ex + mine) {
        unsigned long long acc = ex;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc += qv[j];
          if (acc > target) {
            tok[kstar] = lo + i0 + j;
            sh.found = 1;
            break;
          }
        }
      }
      acc0 += tot_chunk;
      __syncthreads();
      if (sh.found) break;
    }
  }
}

template <int C>
int launch_spec(const SpecParams& p, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows) * C);
  cfg.blockDim = dim3(kSpecThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, spec_accept_kernel<C>, p));
}

template <int C, typename In>
int launch_sampling(const SampParams& p, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(p.per_cta) * sizeof(float);
  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(sampling_kernel<C, In>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSampMaxPerCta * static_cast<int>(sizeof(float)));
    if (e != cudaSuccess) return cuda_status(e);
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows) * C);
  cfg.blockDim = dim3(kSampThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, sampling_kernel<C, In>, p));
}

template <typename In>
int dispatch_cluster(SampParams& p, cudaStream_t s) {
  int c = 1;
  while (c < 8 && (p.vocab + c - 1) / c > kSampMaxPerCta) c <<= 1;
  const int64_t per = ((p.vocab + c - 1) / c + 7) / 8 * 8;  // 16-byte aligned CTA slices
  if (per > kSampMaxPerCta) return INFERD_ERR_UNSUPPORTED;
  p.per_cta = static_cast<int32_t>(per);
  switch (c) {
    case 1: return launch_sampling<1, In>(p, s);
    case 2: return launch_sampling<2, In>(p, s);
    case 4: return launch_sampling<4, In>(p, s);
    default: return launch_sampling<8, In>(p, s);
  }
}

}  // namespace
}  // namespace inferd

using namespace inferd;

extern "C" INFERD_API int inferd_nucleus_sample(float* probs_out, int64_t out_stride, int64_t* tokens,
                                     const void* logits, int32_t dtype, int64_t logits_stride,
                                     int32_t rows, int64_t vocab, const float* temperatures,
                                     float temperature, const float* top_ps, float top_p,
                                     uint64_t seed, uint64_t offset, int32_t* error_word,
                                     void* stream) {
  if (rows < 0 || vocab <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (rows == 0) return INFERD_OK;
  if (!logits || (!probs_out && !tokens)) return INFERD_ERR_INVALID_ARGUMENT;
  if (logits_stride < vocab || (probs_out && out_stride < vocab)) return INFERD_ERR_INVALID_ARGUMENT;
  if (!top_ps && !(top_p > 0.f)) return INFERD_ERR_INVALID_ARGUMENT;  // top_p must be positive
  if (vocab > 0x7fffffff) return INFERD_ERR_UNSUPPORTED;
  SampParams p = {};
  p.src = logits;
  p.stride = logits_stride;
  p.vocab = vocab;
  p.rows = rows;
  p.mode = 0;
  p.temps = temperatures;
  p.temp = temperature;
  p.top_ps = top_ps;
  p.top_p = top_p;
  p.probs_out = probs_out;
  p.out_stride = out_stride;
  p.tokens = tokens;
  p.seed = seed;
  p.offset = offset;
  p.error_word = error_word;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = INFERD_OK;
  if (dtype == INFERD_F32) return dispatch_cluster<float>(p, s);
  if (dtype == INFERD_BF16) return dispatch_nucleus16<__nv_bfloat16>(p, s, &st) ? st : dispatch_cluster<__nv_bfloat16>(p, s);
  if (dtype == INFERD_F16) return dispatch_nucleus16<__half>(p, s, &st) ? st : dispatch_cluster<__half>(p, s);
  return INFERD_ERR_UNSUPPORTED;
}

extern "C" INFERD_API int inferd_sample_probs(int64_t* tokens, const float* probs, int64_t probs_stride, int32_t rows,
                                   int64_t vocab, uint64_t seed, uint64_t offset, int32_t* error_word,
                                   void* stream) {
  if (rows < 0 || vocab <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (rows == 0) return INFERD_OK;
  if (!tokens || !probs || probs_stride < vocab) return INFERD_ERR_INVALID_ARGUMENT;
  if (vocab > 0x7fffffff) return INFERD_ERR_UNSUPPORTED;
  SampParams p = {};
  p.src = probs;
  p.stride = probs_stride;
  p.vocab = vocab;
  p.rows = rows;
  p.mode = 1;
  p.temp = 1.f;
  p.top_p = 1.f;
  p.tokens = tokens;
  p.seed = seed;
  p.offset = offset;
  p.error_word = error_word;
  return dispatch_cluster<float>(p, static_cast<cudaStream_t>(stream));
}

extern "C" INFERD_API int inferd_spec_accept(int32_t* accepted, int64_t* tokens, int64_t tokens_stride,
                                             const float* p, int64_t p_seq_stride, int64_t p_dist_stride,
                                             const float* q, int64_t q_seq_stride, int64_t q_dist_stride,
                                             const int64_t* proposals, int64_t proposals_stride,
                                             int32_t rows, int32_t gamma, int64_t vocab, uint64_t seed,
                                             uint64_t offset, int32_t* error_word, void* stream) {
  if (rows < 0 || gamma < 0 || vocab <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (rows == 0) return INFERD_OK;
  if (!accepted || !tokens || !p || (gamma > 0 && (!q || !proposals))) return INFERD_ERR_INVALID_ARGUMENT;
  if (tokens_stride < gamma + 1 || p_dist_stride < vocab || p_seq_stride < (gamma + 1) * p_dist_stride ||
      (gamma > 0 && (q_dist_stride < vocab || q_seq_stride < gamma * q_dist_stride ||
                     proposals_stride < gamma)))
    return INFERD_ERR_INVALID_ARGUMENT;
  if (vocab > 0x7fffffff) return INFERD_ERR_UNSUPPORTED;
  SpecParams sp = {};
  sp.p = p;
  sp.q = gamma > 0 ? q : p;
  sp.p_row = p_seq_stride;
  sp.p_dist = p_dist_stride;
  sp.q_row = q_seq_stride;
  sp.q_dist = q_dist_stride;
  sp.proposals = gamma > 0 ? proposals : reinterpret_cast<const int64_t*>(tokens);
  sp.prop_row = proposals_stride;
  sp.rows = rows;
  sp.gamma = gamma;
  sp.vocab = vocab;
  sp.accepted = accepted;
  sp.tokens = tokens;
  sp.tok_row = tokens_stride;
  sp.seed = seed;
  sp.offset = offset;
  sp.error_word = error_word;
  // CTAs per sequence: enough to spread a batch over the SMs, each scanning >= 8192 entries
  int c = 1;
  while (c < 8 && static_cast<int64_t>(rows) * c * 2 <= current_sm_count() && vocab / (2 * c) >= 8192) c <<= 1;
  sp.per_cta = static_cast<int32_t>(((vocab + c - 1) / c + 7) / 8 * 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (c) {
    case 1: return launch_spec<1>(sp, s);
    case 2: return launch_spec<2>(sp, s);
    case 4: return launch_spec<4>(sp, s);
    default: return launch_spec<8>(sp, s);
  }
}
