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
__device__ __forceinline__ void block_argmax(SampShared& sh, float& v, int& idx) {
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
__device__ __forceinline__ float block_sum_f32(SampShared& sh, float v) {
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

__device__ __forceinline__ unsigned long long block_sum_u64(SampShared& sh, unsigned long long v) {
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
__device__ __forceinline__ unsigned long long block_exscan_u64(SampShared& sh, unsigned long long v,
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
  if (dtype == INFERD_F32) return dispatch_cluster<float>(p, s);
  if (dtype == INFERD_BF16) return dispatch_cluster<__nv_bfloat16>(p, s);
  if (dtype == INFERD_F16) return dispatch_cluster<__half>(p, s);
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
