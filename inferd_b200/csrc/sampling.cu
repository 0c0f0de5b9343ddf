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
// count and mass.  Masses are summed as round(p * 2^52) integers, so nothing depends on
// the order of atomic updates.  The kept set is every entry whose exclusive cumulative
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
__device__ __forceinline__ uint32_t samp_map(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cl_f32(const void* p, uint32_t rank) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(samp_map(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_cl_u32(const void* p, uint32_t rank) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(samp_map(p, rank)) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_cl_u64(const void* p, uint32_t rank) {
  unsigned long long v;
  asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(v) : "r"(samp_map(p, rank)) : "memory");
  return v;
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
struct SampShared {
  unsigned long long hist_m[256];
  uint32_t hist_c[256];
  unsigned long long tot_m[256];
  uint32_t tot_c[256];
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

// ---------------------------------------------------------------- the kernel
// mode 0: probs_out (optional) = nucleus probabilities; tokens (optional) = one draw.
// mode 1: tokens = one draw from the given non-negative weights (sample_from).
template <int C, typename In>
__global__ void __launch_bounds__(kSampThreads) sampling_kernel(const SampParams p) {
  extern __shared__ __align__(16) float e[];
  __shared__ SampShared sh;
  const int tid = threadIdx.x;
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
  for (int i = tid; i < n; i += kSampThreads) {
    float x = load_src<In>(src + i);
    if (p.mode == 0 && !greedy) x = __fdiv_rn(x, temp);
    if (p.mode == 1 && (!(x >= 0.f) || x == INFINITY)) {  // negative, NaN or infinite weight
      bad = true;
      x = 0.f;
    }
    e[i] = x;
    if (x > mv || (x == mv && static_cast<int>(lo) + i < mi)) {
      mv = x;
      mi = static_cast<int>(lo) + i;
    }
  }
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

  // ---- phase 2: probabilities
  // Fixed point: probabilities (mode 0) as multiples of 2^-52; weights (mode 1) scaled by
  // the power of two 2^(52 - k) with 2^k >= vocab * max weight, so the total stays <= 2^52.
  float fxs = 4503599627370496.0f;
  if (p.mode == 1) {
    int ex = 0;
    frexpf(gmax, &ex);  // gmax <= 2^ex (gmax = 0 gives ex = 0)
    const int lv = p.vocab > 1 ? 64 - __clzll(static_cast<unsigned long long>(p.vocab - 1)) : 0;
    int k = ex + lv;
    if (k < 0) k = 0;
    fxs = ldexpf(1.f, 52 - k);
  }
  unsigned long long total = 0;  // fixed-point mass of every entry
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
    unsigned long long q = 0;
    for (int i = tid; i < n; i += kSampThreads) {
      const float pv = __fdiv_rn(e[i], z);
      e[i] = pv;
      q += to_fixed(pv, fxs);
    }
    q = block_sum_u64(sh, q);
    if (tid == 0) sh.x_u = q;
  } else {
    unsigned long long q = 0;
    for (int i = tid; i < n; i += kSampThreads) q += to_fixed(e[i], fxs);
    if (bad) report_error(p.error_word, INFERD_ERR_INVALID_ARGUMENT);
    q = block_sum_u64(sh, q);
    if (tid == 0) sh.x_u = q;
  }
  samp_cluster_sync();
#pragma unroll
  for (int r = 0; r < C; ++r) total += ld_cl_u64(&sh.x_u, r);
  samp_cluster_sync();

  // ---- phase 3: top-p threshold by radix select on the bits of p
  unsigned long long kept = total;
  const bool cut = p.mode == 0 && top_p < 1.f;
  uint32_t tbits = 0;
  if (cut) {
    const unsigned long long limit = static_cast<unsigned long long>(
        __double2ull_rn(static_cast<double>(top_p) * kFixedOne));
    uint32_t prefix = 0;
    unsigned long long above = 0;
    uint32_t ties = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += kSampThreads) {
        sh.hist_m[b] = 0;
        sh.hist_c[b] = 0;
      }
      __syncthreads();
      const uint32_t hi_mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
      for (int i = tid; i < n; i += kSampThreads) {
        const uint32_t bits = __float_as_uint(e[i]);
        if ((bits & hi_mask) == (prefix & hi_mask)) {
          const uint32_t d = (bits >> shift) & 255u;
          atomicAdd(&sh.hist_m[d], to_fixed(e[i], fxs));
          atomicAdd(&sh.hist_c[d], 1u);
        }
      }
      __syncthreads();
      samp_cluster_sync();  // every CTA's histogram is complete
      for (int b = tid; b < 256; b += kSampThreads) {
        unsigned long long m = 0;
        uint32_t c = 0;
#pragma unroll
        for (int r = 0; r < C; ++r) {
          m += ld_cl_u64(&sh.hist_m[b], r);
          c += ld_cl_u32(&sh.hist_c[b], r);
        }
        sh.tot_m[b] = m;
        sh.tot_c[b] = c;
      }
      samp_cluster_sync();  // remote reads done before the histograms are cleared again
      if (tid == 0) {
        // lowest non-empty bin whose mass above is still within the limit
        unsigned long long acc = above, acc_best = above;
        int best = -1;
        for (int b = 255; b >= 0; --b) {
          if (sh.tot_c[b] > 0) {
            if (acc <= limit) {
              best = b;
              acc_best = acc;
            } else {
              break;
            }
          }
          acc += sh.tot_m[b];
        }
        if (best < 0) best = 0;  // not reached: the largest entry always qualifies
        sh.b_prefix = prefix | (static_cast<uint32_t>(best) << shift);
        sh.b_mass = acc_best;
        sh.b_ties = sh.tot_c[best];
      }
      __syncthreads();
      prefix = sh.b_prefix;
      above = sh.b_mass;
      ties = sh.b_ties;
      __syncthreads();
    }
    tbits = prefix;
    const unsigned long long tq = to_fixed(__uint_as_float(tbits), fxs);
    uint32_t keep_ties = ties;
    if (tq > 0) {
      const unsigned long long room = (limit - above) / tq + 1;  // above <= limit
      if (room < keep_ties) keep_ties = static_cast<uint32_t>(room);
    }
    kept = above + static_cast<unsigned long long>(keep_ties) * tq;

    // ---- phase 4: a tied group cut in the middle keeps its first entries in index order
    if (keep_ties < ties) {
      uint32_t local = 0;
      for (int i = tid; i < n; i += kSampThreads) local += __float_as_uint(e[i]) == tbits ? 1u : 0u;
      local = static_cast<uint32_t>(block_sum_u64(sh, local));
      if (tid == 0) sh.x_u2 = local;
      samp_cluster_sync();
      unsigned long long base = 0;
      for (uint32_t r = 0; r < rank; ++r) base += ld_cl_u64(&sh.x_u2, r);
      samp_cluster_sync();
      for (int c0 = 0; c0 < n; c0 += kSampChunk) {
        const int i0 = c0 + tid * 8;
        uint32_t mine = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i0 + j < n && __float_as_uint(e[i0 + j]) == tbits) ++mine;
        unsigned long long tot_chunk;
        unsigned long long ex = block_exscan_u64(sh, mine, tot_chunk);
        unsigned long long rk = base + ex;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (i0 + j < n && __float_as_uint(e[i0 + j]) == tbits) {
            if (rk >= keep_ties) e[i0 + j] = 0.f;  // dropped: excluded below as p < t
            ++rk;
          }
        base += tot_chunk;
        __syncthreads();
      }
    }
  }

  // ---- phase 5: renormalised probabilities
  if (p.mode == 0 && out) {
    const float s = static_cast<float>(static_cast<double>(kept) / kFixedOne);
    for (int i = tid; i < n; i += kSampThreads) {
      const float v = e[i];
      const bool keep = !cut || __float_as_uint(v) >= tbits;
      out[i] = (keep && v > 0.f) ? __fdiv_rn(v, s) : 0.f;
    }
  }

  // ---- phase 6: one draw, inverse CDF in index order over the kept masses
  if (p.tokens) {
    unsigned long long local = 0;
    for (int i = tid; i < n; i += kSampThreads) {
      const float v = e[i];
      if (!cut || __float_as_uint(v) >= tbits) local += to_fixed(v, fxs);
    }
    local = block_sum_u64(sh, local);
    if (tid == 0) sh.x_u2 = local;
    samp_cluster_sync();
    unsigned long long base = 0;
    for (uint32_t r = 0; r < rank; ++r) base += ld_cl_u64(&sh.x_u2, r);
    samp_cluster_sync();
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
        const unsigned long long ex = base + block_exscan_u64(sh, mine, tot_chunk);
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
        base += tot_chunk;
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
  const int64_t per = (p.vocab + c - 1) / c;
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
