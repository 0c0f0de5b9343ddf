// fp8_linear.cu -- FP8 (e4m3) weight-only linear on tcgen05 tensor cores with TMEM.
//
// y[m, n] = s_w[n] * sum_k x[m, k] * q[n, k]       x bf16 [M, K], q e4m3 [N, K], y bf16 [M, N]
//
// The reference quantises every nn.Linear but lm_head at load time with torchao's
// Float8WeightOnlyConfig (bench/model_loader.py:46-58): per output channel
// s_w[n] = max_k |W[n, k]| / 448 and q = e4m3(W / s_w), activations stay bf16.
//
// tcgen05.mma of kind::f8f6f4 needs both operands in 8-bit formats, and one e4m3 copy of
// a bf16 activation is only ~3 % accurate.  So the activations are split exactly into
// two e4m3 planes under a power-of-two row scale,
//     x[m, k] ~= 2^e[m] * (h[m, k] + l[m, k]),   h = e4m3(x 2^-e),  l = e4m3(x 2^-e - h)
// (about 2^-8 relative per element, the precision of bf16 itself), and both planes are
// multiplied with the same weight tile into one fp32 TMEM accumulator.  The weights are
// read by TMA straight from HBM in their stored e4m3 form; nothing converts them.
//
// Kernel layout (swap-AB): the MMA's M = 128 is the weight rows n, its N is the token
// count m (16..256), so small decode batches do not pad to 128.  One CTA owns 128 weight
// rows: warp 0 streams weight and activation tiles with TMA into a shared-memory ring,
// one thread of warp 1 issues tcgen05.mma and releases stages with tcgen05.commit, and
// all four warps run the epilogue (tcgen05.ld, scale by s_w[n] * 2^e[m], bf16 store).
#include <cuda_fp8.h>

#include <mutex>

#include "common.cuh"
#include "runtime.cuh"

namespace inferd {
namespace {

constexpr int kTileN = 128;     // weight rows per CTA (MMA M)
constexpr int kTileK = 128;     // K bytes per stage = one 128-byte swizzle row
constexpr int kMmaK = 32;       // K per tcgen05.mma of kind::f8f6f4
constexpr int kThreadsFp8 = 128;
constexpr int kMaxTokTile = 256;  // MMA N upper bound
constexpr int kSmemBudget = 200 * 1024;

// ---------------------------------------------------------------- tcgen05 wrappers
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> f32
__device__ __forceinline__ void mma_f8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// mbarrier arrives when every tcgen05.mma issued so far by this thread has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile whose rows are 128 bytes with the
// 128-byte swizzle (8-row atoms of 1024 B): start address, leading byte offset 16 B
// (unused by this layout), stride byte offset 1024 B between 8-row groups, descriptor
// version 1, swizzle mode 2 (128 B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(16u >> 4) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor: kind::f8f6f4, A = B = e4m3, D = f32, both K-major, M = 128.
__host__ __device__ constexpr uint32_t f8_idesc(int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kTileN >> 4) << 24);
}

struct Fp8Params {
  __nv_bfloat16* y;      // [M, N]
  const float* w_scale;  // [N]
  const float* x_scale;  // [M] (powers of two)
  int32_t m, n, k;
  int32_t tok0;          // first token of this launch's token tile
  int32_t tok_tile;      // MMA N (multiple of 16)
  int32_t stages;
  int32_t* error_word;
};

// One CTA = 128 weight rows x tok_tile tokens, full K.
__global__ void __launch_bounds__(kThreadsFp8, 1)
    fp8_linear_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap hmap,
                      const __grid_constant__ CUtensorMap lmap, const Fp8Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[8];
  __shared__ __align__(8) uint64_t empty[8];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kTileN;
  const int T = p.tok_tile;
  const int S = p.stages;
  const uint32_t w_bytes = kTileN * kTileK;  // 16 KiB
  const uint32_t x_bytes = static_cast<uint32_t>(T) * kTileK;
  const uint32_t stage_bytes = w_bytes + 2 * x_bytes;  // multiple of 1024
  const int k_steps = (p.k + kTileK - 1) / kTileK;
  uint32_t ncols = 32;
  while (ncols < static_cast<uint32_t>(T)) ncols <<= 1;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  volatile int* vabort = &abort_flag;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&hmap);
    prefetch_tensormap(&lmap);
    const uint64_t pol_w = l2_policy_evict_first();
    uint64_t pol_x;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_x));
    for (int ks = 0; ks < k_steps; ++ks) {
      const int s = ks % S;
      const uint32_t round = ks / S;
      if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1u)) {
        report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
        *vabort = 1;
        break;
      }
      if (*vabort) break;
      uint8_t* st = smem + s * stage_bytes;
      mbar_arrive_expect_tx(&full[s], stage_bytes);
      tma_load_2d(st, &wmap, ks * kTileK, n0, &full[s], pol_w);
      tma_load_2d(st + w_bytes, &hmap, ks * kTileK, p.tok0, &full[s], pol_x);
      tma_load_2d(st + w_bytes + x_bytes, &lmap, ks * kTileK, p.tok0, &full[s], pol_x);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer (one thread)
    const uint32_t idesc = f8_idesc(T);
    for (int ks = 0; ks < k_steps; ++ks) {
      const int s = ks % S;
      if (*vabort || !mbar_wait(&full[s], (ks / S) & 1u)) {
        report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
        *vabort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t a0 = smem_u32(smem + s * stage_bytes);
      const uint32_t h0 = a0 + w_bytes, l0 = h0 + x_bytes;
#pragma unroll
      for (int kk = 0; kk < kTileK / kMmaK; ++kk) {
        const uint64_t ad = sw128_desc(a0 + kk * kMmaK);
        mma_f8(tmem, ad, sw128_desc(h0 + kk * kMmaK), idesc, (ks | kk) != 0);
        mma_f8(tmem, ad, sw128_desc(l0 + kk * kMmaK), idesc, 1u);
      }
      mma_commit(&empty[s]);  // stage s free once these MMAs have read it
    }
    mma_commit(&acc_full);  // accumulator complete
  }
  __syncwarp();

  // ---------------- epilogue: all four warps, TMEM lanes 32*warp .. 32*warp+31
  bool ok = mbar_wait(&acc_full, 0);
  if (!ok) report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
  tc_fence_after();
  const int n = n0 + warp * 32 + lane;
  const float sw = (ok && n < p.n) ? __ldg(p.w_scale + n) : 0.f;
  for (int c0 = 0; c0 < T; c0 += 16) {
    uint32_t r[16];
    tmem_ld16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, r);
    tmem_ld_wait();
    if (ok && n < p.n) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int m = p.tok0 + c0 + j;
        if (m < p.m) {
          const float v = __uint_as_float(r[j]) * sw * __ldg(p.x_scale + m);
          p.y[static_cast<int64_t>(m) * p.n + n] = __float2bfloat16_rn(v);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
  // never leave with a TMA write in flight: the producer stopped early only on abort,
  // in which case every issued stage was either consumed or is drained here
  if (*vabort && tid == 0) {
    for (int s = 0; s < S && s < k_steps; ++s) {
      const int rounds = (k_steps - s + S - 1) / S;
      mbar_wait(&full[s], (rounds - 1) & 1u);
    }
  }
}

// ---------------------------------------------------------------- activation split
// Row m of x -> e (power-of-two scale), h = e4m3(x 2^-e), l = e4m3(x 2^-e - h).
__device__ __forceinline__ uint8_t to_e4m3(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ float from_e4m3(uint8_t c) {
  const __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(c), __NV_E4M3);
  return __half2float(__half(hr));
}

__global__ void __launch_bounds__(256) split_activations_kernel(const __nv_bfloat16* __restrict__ x, int k,
                                                                uint8_t* __restrict__ h, uint8_t* __restrict__ l,
                                                                float* __restrict__ x_scale) {
  __shared__ float red[8];
  const int m = blockIdx.x;
  const __nv_bfloat16* row = x + static_cast<int64_t>(m) * k;
  float amax = 0.f;
  for (int i = threadIdx.x; i < k; i += blockDim.x) amax = fmaxf(amax, fabsf(__bfloat162float(row[i])));
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
  for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) amax = fmaxf(amax, red[w]);
  // smallest power of two 2^e with amax * 2^-e <= 448: amax = f 2^ex, f in [0.5, 1),
  // 448 = 0.875 * 2^9
  int e = 0;
  if (amax > 0.f) {
    int ex;
    const float f = frexpf(amax, &ex);
    e = ex - 9 + (f > 0.875f ? 1 : 0);
  }
  const float inv = ldexpf(1.f, -e);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    const float v = __bfloat162float(row[i]) * inv;  // exact: power-of-two scaling
    const uint8_t hc = to_e4m3(v);
    const uint8_t lc = to_e4m3(v - from_e4m3(hc));
    h[static_cast<int64_t>(m) * k + i] = hc;
    l[static_cast<int64_t>(m) * k + i] = lc;
  }
  if (threadIdx.x == 0) x_scale[m] = ldexpf(1.f, e);
}

// ---------------------------------------------------------------- weight quantisation
// s[n] = max_k |W[n, k]| / 448 (1 for an all-zero row), q = e4m3(W / s), RN-even.
template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ w, int64_t k,
                                                            uint8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float red[8];
  const int64_t n = blockIdx.x;
  const T* row = w + n * k;
  float amax = 0.f;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) amax = fmaxf(amax, fabsf(to_f32<T>(row[i])));
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) amax = fmaxf(amax, red[i]);
  float s = __fdiv_rn(amax, 448.f);
  if (!(s > 0.f)) s = 1.f;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) q[n * k + i] = to_e4m3(__fdiv_rn(to_f32<T>(row[i]), s));
  if (threadIdx.x == 0) scale[n] = s;
}

// ---------------------------------------------------------------- host side
inline int encode_u8_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                         uint32_t box_rows) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return INFERD_ERR_CUDA;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? INFERD_OK : INFERD_ERR_CUDA;
}

inline size_t align256_fp8(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct Fp8Workspace {
  size_t h, l, scale, total;
};
inline Fp8Workspace fp8_workspace(int64_t m, int64_t k) {
  Fp8Workspace w;
  w.h = 0;
  w.l = align256_fp8(static_cast<size_t>(m * k));
  w.scale = w.l + align256_fp8(static_cast<size_t>(m * k));
  w.total = w.scale + align256_fp8(static_cast<size_t>(m) * 4);
  return w;
}

}  // namespace
}  // namespace inferd

using namespace inferd;

extern "C" size_t inferd_fp8_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int32_t device) {
  (void)n;
  (void)device;
  if (m <= 0 || k <= 0) return 0;
  return fp8_workspace(m, k).total;
}

extern "C" int inferd_fp8_quantize_per_channel(const void* w, int32_t w_dtype, void* w_e4m3, float* w_scale,
                                               int64_t n, int64_t k, void* stream) {
  if (n < 0 || k <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (n == 0) return INFERD_OK;
  if (!w || !w_e4m3 || !w_scale) return INFERD_ERR_INVALID_ARGUMENT;
  if (n > 0x7fffffff) return INFERD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(static_cast<unsigned>(n));
  if (w_dtype == INFERD_BF16)
    quantize_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(w), k,
                                                             static_cast<uint8_t*>(w_e4m3), w_scale);
  else if (w_dtype == INFERD_F16)
    quantize_rows_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(w), k,
                                                      static_cast<uint8_t*>(w_e4m3), w_scale);
  else if (w_dtype == INFERD_F32)
    quantize_rows_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(w), k,
                                                     static_cast<uint8_t*>(w_e4m3), w_scale);
  else
    return INFERD_ERR_UNSUPPORTED;
  return launch_status();
}

extern "C" int inferd_fp8_linear(void* y, const void* x, const void* w_e4m3, const float* w_scale, int64_t m,
                                 int64_t n, int64_t k, void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 0 || n <= 0 || k <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (m == 0) return INFERD_OK;
  if (!y || !x || !w_e4m3 || !w_scale) return INFERD_ERR_INVALID_ARGUMENT;
  if (k % 16 != 0) return INFERD_ERR_UNSUPPORTED;  // TMA rows must be 16-byte multiples
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return INFERD_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(w_e4m3) & 15) != 0) return INFERD_ERR_INVALID_ARGUMENT;
  const Fp8Workspace wl = fp8_workspace(m, k);
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0 || workspace_bytes < wl.total)
    return INFERD_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* h = ws + wl.h;
  uint8_t* l = ws + wl.l;
  float* xs = reinterpret_cast<float*>(ws + wl.scale);

  split_activations_kernel<<<static_cast<unsigned>(m), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x),
                                                                   static_cast<int>(k), h, l, xs);
  int st = launch_status();
  if (st != INFERD_OK) return st;

  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(fp8_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 1024);
    if (e != cudaSuccess) return cuda_status(e);
    configured[dev] = true;
  }

  CUtensorMap wmap;
  st = encode_u8_map(&wmap, w_e4m3, static_cast<uint64_t>(n), static_cast<uint64_t>(k), kTileN);
  if (st != INFERD_OK) return st;
  const unsigned grid = static_cast<unsigned>((n + kTileN - 1) / kTileN);
  for (int64_t t0 = 0; t0 < m; t0 += kMaxTokTile) {
    const int64_t rem = m - t0;
    const int tile = static_cast<int>(((rem < kMaxTokTile ? rem : kMaxTokTile) + 15) / 16 * 16);
    CUtensorMap hmap, lmap;
    st = encode_u8_map(&hmap, h, static_cast<uint64_t>(m), static_cast<uint64_t>(k), static_cast<uint32_t>(tile));
    if (st != INFERD_OK) return st;
    st = encode_u8_map(&lmap, l, static_cast<uint64_t>(m), static_cast<uint64_t>(k), static_cast<uint32_t>(tile));
    if (st != INFERD_OK) return st;
    const int stage_bytes = kTileN * kTileK + 2 * tile * kTileK;
    int stages = kSmemBudget / stage_bytes;
    if (stages > 8) stages = 8;
    if (stages < 2) return INFERD_ERR_UNSUPPORTED;
    Fp8Params p;
    p.y = static_cast<__nv_bfloat16*>(y);
    p.w_scale = w_scale;
    p.x_scale = xs;
    p.m = static_cast<int32_t>(m);
    p.n = static_cast<int32_t>(n);
    p.k = static_cast<int32_t>(k);
    p.tok0 = static_cast<int32_t>(t0);
    p.tok_tile = tile;
    p.stages = stages;
    p.error_word = nullptr;
    const size_t smem = 1024 + static_cast<size_t>(stages) * stage_bytes;
    fp8_linear_kernel<<<grid, kThreadsFp8, smem, s>>>(wmap, hmap, lmap, p);
    st = launch_status();
    if (st != INFERD_OK) return st;
  }
  return INFERD_OK;
}
