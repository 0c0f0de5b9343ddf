// fp8_linear.cu -- FP8 (e4m3) weight-only linear on tcgen05 tensor cores with TMEM.
//
// y[m, n] = s_w[n] * sum_k x[m, k] * q[n, k]       x bf16 [M, K], q e4m3 [N, K], y bf16 [M, N]
//
// The same GEMM serves the reference's "fp8-dynamic" recipe (torchao's
// Float8DynamicActivationFloat8WeightConfig, bench/model_loader.py:53-55): there x is
// quantised on the fly to ONE e4m3 plane with s_x = amax / 448 (per tensor or per row) and
// y = s_x[m] s_w[n] sum_k q_x[m, k] q[n, k] -- the kernel's `planes = 1` mode.
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
// Weight layouts.  Row-major [N, K] e4m3 is read by TMA 128 bytes per row per stage.
// The packed layout produced once at load time stores every 128-row x 128-byte tile as
// one contiguous 16 KiB block, already in the 128-byte-swizzled shared-memory form the
// MMA reads, tiles of one 128-row band consecutive along K, bands padded to an even
// count -- so each CTA streams one contiguous region, copied verbatim by TMA as 128-byte
// rows.  Tiles past N or K are zero-filled.
//
// Kernel layout (swap-AB, CTA pairs): the MMA's M is the weight rows and its N the token
// count m (16..256), so small decode batches do not pad to 128.  Two CTAs on two SMs form
// a cluster that issues tcgen05.mma.cta_group::2 with M = 256: each CTA holds its own
// 128-row weight tile and half of the activation tile, which halves the activation bytes
// every SM stages per weight byte.  Per CTA, warp 0 streams tiles with TMA into a
// shared-memory ring, one thread of the leader CTA's warp 1 issues the MMAs and releases
// stages of both CTAs with tcgen05.commit, and four epilogue warps drain double-buffered
// TMEM accumulators (tcgen05.ld, scale by s_w[n] * 2^e[m]) into y with TMA stores.
#include <cuda_fp8.h>

#include <cstring>
#include <mutex>

#include "common.cuh"
#include "runtime.cuh"

namespace inferd {
namespace {

constexpr int kTileN = 128;     // weight rows per CTA (MMA M)
constexpr int kTileK = 128;     // K bytes per stage = one 128-byte swizzle row
constexpr int kMmaK = 32;       // K per tcgen05.mma of kind::f8f6f4
constexpr int kMaxTokTile = 256;  // MMA N upper bound
constexpr int kSmemBudget = 224 * 1024;   // one CTA per SM
constexpr int kSmemBudget2 = 108 * 1024;  // two CTAs per SM
// epilogue shared memory after the ring: per epilogue warp four 16-token x 32-row bf16
// blocks (two per 32-token step, double-buffered), then the launch tile's token scales
constexpr int kEpiBlockElems = 16 * 32;
constexpr int kEpiStageBytes = 4 * 4 * kEpiBlockElems * 2 + kMaxTokTile * 4;

// ---------------------------------------------------------------- tcgen05 / cluster wrappers
// Every tcgen05 instruction of the GEMM uses .cta_group::2: the two CTAs of a cluster
// form one 256-row MMA (each CTA holds its 128 weight rows as A and half of the B rows).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T over the CTA pair, e4m3 x e4m3 -> f32
__device__ __forceinline__ void mma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The mbarrier at the same shared-memory offset in both CTAs of the pair receives one
// arrival once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// all threads of both CTAs; orders shared-memory writes (barrier inits) cluster-wide
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of this CTA's variable at `smem_addr` as seen in CTA `rank`
__device__ __forceinline__ uint32_t cluster_addr(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory; the bytes are counted on the mbarrier
// at bar_cluster_addr, which may be the peer CTA's (.cta_group::2)
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                                 uint32_t bar_cluster_addr, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster_addr), "l"(policy)
      : "memory");
}
// 2-D tiled TMA store from this CTA's shared memory (bulk async-group completion); rows
// and columns outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int32_t c0, int32_t c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most one committed store group still reads shared memory
__device__ __forceinline__ void bulk_wait_read_le1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Instruction descriptor: kind::f8f6f4, A = B = e4m3, D = f32, both K-major, M = 256 (the
// CTA pair), N = n.
__host__ __device__ constexpr uint32_t f8_idesc_pair(int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(256 >> 4) << 24);
}

struct Fp8Params {
  __nv_bfloat16* y;         // [M, N]
  const float* w_scale;     // [N]
  const float* x_scale;     // [M] (powers of two)
  int32_t m, n, k;
  int32_t w_packed;         // 1: wmap views the packed tiles as [tiles * 128 rows, 128 B]
  int32_t tok0;             // first token of this launch's token tile
  int32_t tok_tile;         // tokens per launch tile T (multiple of 16)
  int32_t stages;
  int32_t* counters;        // [weight tiles] tickets, 0 between launches
  float* part;              // [slot][2][T][128] partial accumulators
  int32_t* error_word;
  int32_t y_tma;            // 1: ymap describes y (bf16 [M, N], 16-byte row pitch)
  int32_t planes;           // activation planes: 2 = exact h + l split, 1 = one e4m3 copy
};

constexpr int kFp8Warps = 6;  // 0: TMA producer, 1: MMA issuer (leader CTA), 2..5: epilogue
constexpr int kFp8Threads = kFp8Warps * 32;

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 lane;\n\t.reg .pred p;\n\t"
      "elect.sync lane|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

// Cluster whose balanced range [c*W/C, (c+1)*W/C) of the work axis contains unit g.
__device__ __forceinline__ int fp8_cluster_of(int64_t g, int64_t W, int C) {
  int64_t c = ((g + 1) * C + W - 1) / W - 1;
  if (c < 0) c = 0;
  if (c > C - 1) c = C - 1;
  return static_cast<int>(c);
}

// B rows each CTA of the pair holds for a launch tile of T tokens.  Two planes (the exact
// split): with T <= 128 the MMA's B operand is [h tile; l tile] (N = 2T): CTA 0 holds the
// h plane, CTA 1 the l plane, and the accumulator's column halves are added in the
// epilogue.  With T > 128 (N would exceed 256) the h and l MMAs (N = T each) accumulate
// into the same T columns and each CTA holds T/2 tokens of both planes.  Either way a CTA
// stages T * 128 activation bytes per K step.  One plane (dynamic activation scaling):
// N = T, each CTA holds T/2 tokens, T/2 * 128 bytes per K step.
__host__ __device__ constexpr int fp8_acc_cols(int T, int planes) { return planes == 2 && T <= 128 ? 2 * T : T; }
__host__ __device__ constexpr int fp8_x_stage_bytes(int T, int planes) {
  return planes == 2 ? T * kTileK : (T / 2) * kTileK;
}
// tcgen05.alloc takes a power of two >= 32; two accumulators (double buffering)
__host__ __device__ constexpr uint32_t fp8_tmem_cols(int T, int planes) {
  uint32_t c = 32;
  while (c < static_cast<uint32_t>(2 * fp8_acc_cols(T, planes))) c <<= 1;
  return c;
}

// One cluster of two CTAs (on two SMs) computes weight-tile pairs: tile pair tp is weight
// rows [256 tp, 256 tp + 256), CTA r of the pair owns tile t = 2 tp + r.  Stream-K over the
// work axis (tile pair, K step) -> g = tp * KS + ks: cluster c of C runs [c*W/C, (c+1)*W/C).
// Every run of one tile pair inside that range is a segment with its own accumulator;
// segments alternate between two TMEM accumulators, so the MMA warp starts the next
// segment while the epilogue drains the previous one.  A segment covering a whole tile is
// stored directly.  Otherwise the pieces of a tile are merged by the CTA that finishes it
// last: straight from its TMEM when the sibling pieces are already stored (the usual case
// at the end of a range), or from the stored partials.
//
// Pipeline.  Each CTA's producer streams its own weight tile and its half of the
// activation tile into its ring; both CTAs' loads count on the leader CTA's full barrier.
// The leader's MMA warp issues the pair MMAs and commits to the empty barriers of both
// CTAs (and to both CTAs' accumulator barriers at the end of a segment); each CTA's four
// epilogue warps read their own TMEM lanes, arrive on the leader's acc_empty barrier and
// write y through shared memory with TMA stores.
__global__ void __launch_bounds__(kFp8Threads, 2)
    fp8_linear_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap hmap,
                      const __grid_constant__ CUtensorMap lmap, const __grid_constant__ CUtensorMap ymap,
                      const Fp8Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full[8];
  __shared__ __align__(8) uint64_t empty[8];
  __shared__ __align__(8) uint64_t acc_full[2];
  __shared__ __align__(8) uint64_t acc_empty[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ int last_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int T = p.tok_tile;
  const int S = p.stages;
  const bool two = p.planes == 2;
  const bool merged = two && T <= 128;
  const uint32_t w_bytes = kTileN * kTileK;                                        // 16 KiB
  const uint32_t x_bytes = static_cast<uint32_t>(fp8_x_stage_bytes(T, p.planes));  // this CTA's activation rows
  const uint32_t stage_bytes = w_bytes + x_bytes;              // multiple of 1024
  const int KS = (p.k + kTileK - 1) / kTileK;
  const int NT = (p.n + kTileN - 1) / kTileN;
  const int NP = (NT + 1) / 2;
  const int64_t W = static_cast<int64_t>(NP) * KS;
  const int C = gridDim.x / 2;
  const int cl = blockIdx.x / 2;
  const int64_t g0 = static_cast<int64_t>(cl) * W / C;
  const int64_t g1 = static_cast<int64_t>(cl + 1) * W / C;
  const int n_units = static_cast<int>(g1 - g0);
  const uint32_t acc_cols = static_cast<uint32_t>(fp8_acc_cols(T, p.planes));
  const uint32_t ncols = fp8_tmem_cols(T, p.planes);

  if (tid == 0) {
    // descriptor fetches overlap the set-up below
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&hmap);
    if (p.planes == 2) prefetch_tensormap(&lmap);
    if (p.y_tma) prefetch_tensormap(&ymap);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);  // one arrival per epilogue warp of both CTAs
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&tmem_base, ncols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barrier inits and the TMEM address are visible to both CTAs
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  volatile int* vabort = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      const uint64_t pol_w = l2_policy_evict_first();
      uint64_t pol_x;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_x));
      const int x_row = merged ? p.tok0 : p.tok0 + static_cast<int>(rank) * (T / 2);
      // Work unit g0 + j is (tile pair tp, K step ks); both advance with the loop, so no
      // unit pays for a 64-bit division.
      const int tp0 = static_cast<int>(g0 / KS);
      const int ks0 = static_cast<int>(g0 - static_cast<int64_t>(tp0) * KS);
      auto load_w = [&](uint8_t* st, int tp, int ks, uint32_t bar) {
        const int t = 2 * tp + static_cast<int>(rank);
        if (p.w_packed) tma_load_2d_pair(st, &wmap, 0, (t * KS + ks) * kTileN, bar, pol_w);
        else tma_load_2d_pair(st, &wmap, ks * kTileK, t * kTileN, bar, pol_w);
      };
      auto load_x = [&](uint8_t* st, int ks, uint32_t bar) {
        if (merged) {
          tma_load_2d_pair(st + w_bytes, leader ? &hmap : &lmap, ks * kTileK, x_row, bar, pol_x);
        } else if (two) {
          tma_load_2d_pair(st + w_bytes, &hmap, ks * kTileK, x_row, bar, pol_x);
          tma_load_2d_pair(st + w_bytes + x_bytes / 2, &lmap, ks * kTileK, x_row, bar, pol_x);
        } else {
          tma_load_2d_pair(st + w_bytes, &hmap, ks * kTileK, x_row, bar, pol_x);
        }
      };
      auto full_of = [&](int s) { return cluster_addr(smem_u32(&full[s]), 0); };
      // The weight tiles of the first ring do not depend on the activation split: issue
      // them before waiting for it.
      const int first = n_units < S ? n_units : S;
      int tp = tp0, ks = ks0;
      for (int j = 0; j < first; ++j) {
        if (leader) mbar_arrive_expect_tx(&full[j], 2 * stage_bytes);
        load_w(smem + j * stage_bytes, tp, ks, full_of(j));
        if (++ks == KS) { ks = 0; ++tp; }
      }
      grid_dependency_wait();
      ks = ks0;
      for (int j = 0; j < first; ++j) {
        load_x(smem + j * stage_bytes, ks, full_of(j));
        if (++ks == KS) ks = 0;
      }
      // from unit S on: stage s = j % S, refilled once its previous fill (parity
      // j / S - 1) has been consumed
      int s = 0;
      uint32_t par = 0;
      for (int j = first; j < n_units; ++j) {
        if (*vabort) break;
        if (!mbar_wait(&empty[s], par)) {
          report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
          *vabort = 1;
          break;
        }
        uint8_t* st = smem + s * stage_bytes;
        if (leader) mbar_arrive_expect_tx(&full[s], 2 * stage_bytes);
        load_w(st, tp, ks, full_of(s));
        load_x(st, ks, full_of(s));
        if (++ks == KS) { ks = 0; ++tp; }
        if (++s == S) { s = 0; par ^= 1u; }
      }
      // every load of this CTA is issued: the next call's first kernel may launch (it
      // waits for this grid to finish before it touches anything this grid reads)
      grid_launch_dependents();
    }
    __syncwarp();
  } else if (warp == 1) {
    if (leader) {
      // ---------------- MMA issuer: the whole warp walks the loop, one elected lane issues
      const uint32_t idesc = f8_idesc_pair(merged ? 2 * T : T);
      int seg = 0;        // segments started
      int in_seg = 0;     // K steps issued in the current segment
      uint32_t acc = tmem;
      int ks = static_cast<int>(g0 % KS);  // K step of unit j, advanced with the loop
      int s = 0;                           // its stage, j % S, and the fill's parity
      uint32_t par = 0;
      for (int j = 0; j < n_units; ++j) {
        const bool seg_begin = (j == 0) || (ks == 0);
        const bool seg_end = (j == n_units - 1) || (ks == KS - 1);
        // Waits are done by lane 0 and broadcast, so every branch below is warp-uniform
        // (elect.sync needs the whole warp).
        if (seg_begin) {
          const int buf = seg & 1;
          // this buffer's previous segment (two back) must have been read out by both CTAs
          if (seg >= 2) {
            int w_ok = 1;
            if (lane == 0 && !*vabort) {
              w_ok = mbar_wait(&acc_empty[buf], ((seg >> 1) - 1) & 1u) ? 1 : 0;
              if (!w_ok) {
                report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
                *vabort = 1;
              }
            }
            __shfl_sync(0xffffffffu, w_ok, 0);
          }
          acc = tmem + static_cast<uint32_t>(buf) * acc_cols;
          in_seg = 0;
          tc_fence_after();
        }
        int ok = 0;
        if (lane == 0 && !*vabort) {
          ok = mbar_wait(&full[s], par) ? 1 : 0;
          if (!ok) {
            report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
            *vabort = 1;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (ok && elect_one()) {
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem + s * stage_bytes);
          const uint32_t b0 = a0 + w_bytes;
#pragma unroll
          for (int kk = 0; kk < kTileK / kMmaK; ++kk) {
            const uint64_t ad = sw128_desc(a0 + kk * kMmaK);
            const uint32_t accumulate = (in_seg | kk) != 0 ? 1u : 0u;
            mma_f8_pair(acc, ad, sw128_desc(b0 + kk * kMmaK), idesc, accumulate);
            if (two && !merged) mma_f8_pair(acc, ad, sw128_desc(b0 + x_bytes / 2 + kk * kMmaK), idesc, 1u);
          }
          mma_commit_pair(&empty[s]);  // stage s free in both CTAs once these MMAs have read it
        }
        __syncwarp();
        ++in_seg;
        if (seg_end) {
          if (elect_one()) mma_commit_pair(&acc_full[seg & 1]);  // segment accumulator complete
          __syncwarp();
          ++seg;
        }
        if (++ks == KS) ks = 0;
        if (++s == S) { s = 0; par ^= 1u; }
      }
    }
  } else {
    // ---------------- epilogue warps 2..5 (both CTAs): TMEM lane quarter q = warp % 4
    const int q = warp & 3;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const int ep = tid - 64;  // 0..127 among the epilogue threads
    const int row = q * 32 + lane;
    // per-warp output staging for the TMA stores, and the launch tile's token scales
    __nv_bfloat16* ystage = reinterpret_cast<__nv_bfloat16*>(smem + S * stage_bytes) + (warp - 2) * 4 * kEpiBlockElems;
    float* xsm = reinterpret_cast<float*>(smem + S * stage_bytes + 4 * 4 * kEpiBlockElems * 2);
    int ychunk = 0;  // store groups committed by this warp
    grid_dependency_wait();  // x_scale comes from the split grid
    for (int i = ep; i < T; i += 128) xsm[i] = p.tok0 + i < p.m ? __ldg(p.x_scale + p.tok0 + i) : 0.f;
    named_barrier_sync(1, 128);
    int seg = 0;
    int64_t g = g0;
    while (g < g1) {
      const int tp = static_cast<int>(g / KS);
      const int t = 2 * tp + static_cast<int>(rank);
      const int64_t t_begin = static_cast<int64_t>(tp) * KS, t_end = t_begin + KS;
      const int64_t s_end = g1 < t_end ? g1 : t_end;
      const bool whole = (g == t_begin) && (s_end == t_end);
      const int buf = seg & 1;
      bool ok = !*vabort && mbar_wait(&acc_full[buf], (seg >> 1) & 1u);
      if (!ok && !*vabort) {
        report_error(p.error_word, INFERD_ERR_DEVICE_TIMEOUT);
        *vabort = 1;
      }
      tc_fence_after();
      const uint32_t acc = lane_base + static_cast<uint32_t>(buf) * acc_cols;
      const int n_idx = t * kTileN + row;
      const float sw = (n_idx < p.n) ? __ldg(p.w_scale + n_idx) : 0.f;
      const int c_first = whole ? cl : fp8_cluster_of(t_begin, W, C);
      const int c_last = whole ? cl : fp8_cluster_of(t_end - 1, W, C);
      // A partial segment whose sibling pieces are all stored already is merged straight
      // from TMEM, without storing and re-reading its own piece.
      bool merge_now = whole;
      if (!whole) {
        if (ep == 0) last_flag = atomicAdd(p.counters + t, 0) == c_last - c_first ? 1 : 0;
        named_barrier_sync(1, 128);
        merge_now = last_flag != 0;
        if (merge_now) __threadfence();
      }
      if (merge_now) {
        // y = s_w * 2^e * (own accumulator + the stored sibling pieces), 32 tokens per step
        for (int c0 = 0; c0 < T; c0 += 32) {
          const bool wide = T - c0 >= 32;
          uint32_t vr[32];  // accumulator values (fp32 bits)
          {
            uint32_t rl[32];
            if (wide) {
              tmem_ld32(acc + static_cast<uint32_t>(c0), vr);
              if (merged) tmem_ld32(acc + static_cast<uint32_t>(T + c0), rl);
            } else {
              tmem_ld16(acc + static_cast<uint32_t>(c0), vr);
              if (merged) tmem_ld16(acc + static_cast<uint32_t>(T + c0), rl);
            }
            tmem_ld_wait();
            if (merged) {
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) vr[jj] = __float_as_uint(__uint_as_float(vr[jj]) + __uint_as_float(rl[jj]));
            }
          }
          float* v = reinterpret_cast<float*>(vr);
          if (!whole) {
            for (int cc = c_first; cc <= c_last; ++cc) {
              if (cc == cl) continue;
              const float* src = p.part + (2 * (static_cast<int64_t>(cc) + tp) + rank) * T * kTileN +
                                 static_cast<int64_t>(c0) * kTileN + row;
#pragma unroll
              for (int jj = 0; jj < 32; ++jj)
                if (jj < 16 || wide) v[jj] += __ldcg(src + jj * kTileN);
            }
          }
          // the chunk's 32 token scales (entries past the tile are never stored)
          const float4* xs4 = reinterpret_cast<const float4*>(xsm + c0);
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const float4 f = xs4[i4];
            v[4 * i4 + 0] *= sw * f.x;
            v[4 * i4 + 1] *= sw * f.y;
            v[4 * i4 + 2] *= sw * f.z;
            v[4 * i4 + 3] *= sw * f.w;
          }
          const int n0 = t * kTileN + q * 32, m0 = p.tok0 + c0;
          if (p.y_tma) {
            if (n0 < p.n && m0 < p.m) {
              // a [32 tokens][32 rows] block of y in shared memory, then one TMA store (a
              // 16-token chunk only occurs at the end of the last launch tile, where the
              // tensor map clips the block's rows past M)
              __nv_bfloat16* blk = ystage + (ychunk & 1) * 2 * kEpiBlockElems;
              if (lane == 0) bulk_wait_read_le1();  // the group that last read these blocks is done
              __syncwarp();
#pragma unroll
              for (int jj = 0; jj < 32; ++jj)
                if (jj < 16 || wide) blk[jj * 32 + lane] = __float2bfloat16_rn(v[jj]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&ymap, blk, n0, m0);
                bulk_commit_group();
              }
              ++ychunk;
            }
          } else if (n_idx < p.n) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const int m = m0 + jj;
              if ((jj < 16 || wide) && m < p.m) p.y[static_cast<int64_t>(m) * p.n + n_idx] = __float2bfloat16_rn(v[jj]);
            }
          }
        }
        if (!whole && ep == 0) p.counters[t] = 0;
      } else {
        const int64_t slot = 2 * (static_cast<int64_t>(cl) + tp) + rank;
        float* prow = p.part + slot * static_cast<int64_t>(T) * kTileN + row;
        for (int c0 = 0; c0 < T; c0 += 16) {
          uint32_t rh[16], rl[16];
          tmem_ld16(acc + static_cast<uint32_t>(c0), rh);
          if (merged) tmem_ld16(acc + static_cast<uint32_t>(T + c0), rl);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj)
            prow[static_cast<int64_t>(c0 + jj) * kTileN] =
                merged ? __uint_as_float(rh[jj]) + __uint_as_float(rl[jj]) : __uint_as_float(rh[jj]);
        }
      }
      // accumulator read out: the leader's MMA warp may reuse this buffer
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(smem_u32(&acc_empty[buf]), 0));
      if (!merge_now) {
        __threadfence();
        named_barrier_sync(1, 128);
        if (ep == 0) {
          const int prev = atomicAdd(p.counters + t, 1);
          last_flag = (prev == c_last - c_first) ? 1 : 0;
        }
        named_barrier_sync(1, 128);
        if (last_flag) {
          __threadfence();
          // the siblings finished meanwhile: merge every piece, this one included
          for (int c0 = 0; c0 < T; c0 += 16) {
            float sum[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) sum[jj] = 0.f;
            for (int cc = c_first; cc <= c_last; ++cc) {
              const float* src = p.part + (2 * (static_cast<int64_t>(cc) + tp) + rank) * T * kTileN +
                                 static_cast<int64_t>(c0) * kTileN + row;
              float o[16];
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) o[jj] = __ldcg(src + jj * kTileN);
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) sum[jj] += o[jj];
            }
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) {
              const int m = p.tok0 + c0 + jj;
              if (m < p.m && n_idx < p.n)
                p.y[static_cast<int64_t>(m) * p.n + n_idx] = __float2bfloat16_rn(sum[jj] * sw * xsm[c0 + jj]);
            }
          }
          if (ep == 0) p.counters[t] = 0;
        }
      }
      named_barrier_sync(1, 128);  // last_flag is rewritten by the next segment
      ++seg;
      g = s_end;
    }
    // the CTA may retire once its store groups have read their shared-memory blocks; the
    // global writes complete with the grid
    if (lane == 0 && ychunk > 0) bulk_wait_read_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // never leave with a TMA write in flight (only possible after an abort): both CTAs'
  // bytes count on the leader's full barriers
  if (leader && tid == 0 && *vabort) {
    for (int s = 0; s < S && s < n_units; ++s) {
      const int rounds = (n_units - s + S - 1) / S;
      mbar_wait(&full[s], (rounds - 1) & 1u);
    }
  }
  // neither CTA leaves while the pair's MMAs or loads may still touch its shared memory
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, ncols);
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

// One CTA per token row.  Each thread holds up to kSplitRegs groups of 8 bf16 in registers
// (16-byte loads), so the row is read from global memory once when K <= 256 * 8 * 4.
constexpr int kSplitThreads = 256;
constexpr int kSplitRegs = 4;

__device__ __forceinline__ uint32_t split_pair(float a, float b, uint32_t& lo_out) {
  // returns h codes of (a, b) in the low 16 bits; l codes in lo_out
  const uint8_t ha = to_e4m3(a), hb = to_e4m3(b);
  const uint8_t la = to_e4m3(a - from_e4m3(ha)), lb = to_e4m3(b - from_e4m3(hb));
  lo_out = static_cast<uint32_t>(la) | (static_cast<uint32_t>(lb) << 8);
  return static_cast<uint32_t>(ha) | (static_cast<uint32_t>(hb) << 8);
}

__global__ void __launch_bounds__(kSplitThreads) split_activations_kernel(const __nv_bfloat16* __restrict__ x, int k,
                                                                         uint8_t* __restrict__ h, uint8_t* __restrict__ l,
                                                                         float* __restrict__ x_scale) {
  __shared__ float red[kSplitThreads / 32];
  // Launched early (programmatic dependent launch): x and the workspace planes may belong
  // to the previous grid until it completes, so nothing is read or written before the
  // wait.  The GEMM may launch at once: before its own wait it only loads weights, which no
  // grid of this library writes (weights are written by load-time kernels that never
  // trigger early), so its prologue and first weight ring overlap the previous call's tail.
  grid_launch_dependents();
  grid_dependency_wait();
  const int m = blockIdx.x;
  const __nv_bfloat16* row = x + static_cast<int64_t>(m) * k;
  const int groups = k / 8;  // k % 16 == 0
  uint4 keep[kSplitRegs];
  float amax = 0.f;
#pragma unroll
  for (int r = 0; r < kSplitRegs; ++r) {
    const int gidx = threadIdx.x + r * kSplitThreads;
    keep[r] = make_uint4(0, 0, 0, 0);
    if (gidx < groups) keep[r] = __ldg(reinterpret_cast<const uint4*>(row) + gidx);
  }
  auto group_max = [](const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a = fmaxf(a, fabsf(__uint_as_float(w[j] << 16)));
      a = fmaxf(a, fabsf(__uint_as_float(w[j] & 0xffff0000u)));
    }
    return a;
  };
#pragma unroll
  for (int r = 0; r < kSplitRegs; ++r) amax = fmaxf(amax, group_max(keep[r]));
  for (int gidx = threadIdx.x + kSplitRegs * kSplitThreads; gidx < groups; gidx += kSplitThreads)
    amax = fmaxf(amax, group_max(*reinterpret_cast<const uint4*>(row + gidx * 8)));
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
  for (int w = 0; w < kSplitThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  // smallest power of two 2^e with amax * 2^-e <= 448: amax = f 2^ex, f in [0.5, 1),
  // 448 = 0.875 * 2^9
  int e = 0;
  if (amax > 0.f) {
    int ex;
    const float f = frexpf(amax, &ex);
    e = ex - 9 + (f > 0.875f ? 1 : 0);
  }
  const float inv = ldexpf(1.f, -e);
  auto emit = [&](const uint4& v, int gidx) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t l0, l1;
      // exact: power-of-two scaling of bf16 values
      const uint32_t h0 = split_pair(__uint_as_float(w[2 * half] << 16) * inv,
                                     __uint_as_float(w[2 * half] & 0xffff0000u) * inv, l0);
      const uint32_t h1 = split_pair(__uint_as_float(w[2 * half + 1] << 16) * inv,
                                     __uint_as_float(w[2 * half + 1] & 0xffff0000u) * inv, l1);
      hw[half] = h0 | (h1 << 16);
      lw[half] = l0 | (l1 << 16);
    }
    const int64_t off = static_cast<int64_t>(m) * k + gidx * 8;
    *reinterpret_cast<uint2*>(h + off) = make_uint2(hw[0], hw[1]);
    *reinterpret_cast<uint2*>(l + off) = make_uint2(lw[0], lw[1]);
  };
#pragma unroll
  for (int r = 0; r < kSplitRegs; ++r) {
    const int gidx = threadIdx.x + r * kSplitThreads;
    if (gidx < groups) emit(keep[r], gidx);
  }
  for (int gidx = threadIdx.x + kSplitRegs * kSplitThreads; gidx < groups; gidx += kSplitThreads)
    emit(*reinterpret_cast<const uint4*>(row + gidx * 8), gidx);
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

// ---------------------------------------------------------------- dynamic (absmax) scaling
// torchao's Float8DynamicActivationFloat8WeightConfig scales a tensor by s = amax / 448,
// over the whole tensor (PerTensor, its default) or per row (PerRow), and stores
// q = e4m3(clamp(x / s, -448, 448)); the same rule quantises the activations of every
// forward and, once, the weights.  amax is exact (a maximum of magnitudes), s an fp32
// division, x / s an IEEE division rounded to fp32, the cast round-to-nearest-even with
// saturation (the clamp).  An all-zero tensor (row) gets s = 1 and zero codes.

// 16-byte vector loads over a row of T when its length and base allow them.
template <typename T>
__device__ __forceinline__ bool row_vectorizable(const T* row, int64_t k) {
  return (k * static_cast<int64_t>(sizeof(T))) % 16 == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0;
}
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float* out) {
  constexpr int E = 16 / sizeof(T);
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int j = 0; j < E; ++j) out[j] = to_f32<T>(e[j]);
}

template <typename T>
__device__ float row_absmax(const T* __restrict__ row, int64_t k, float* red) {
  constexpr int E = 16 / sizeof(T);
  float amax = 0.f;
  if (row_vectorizable(row, k)) {
    const uint4* v = reinterpret_cast<const uint4*>(row);
    for (int64_t i = threadIdx.x; i < k / E; i += blockDim.x) {
      float f[E];
      unpack16<T>(__ldg(v + i), f);
#pragma unroll
      for (int j = 0; j < E; ++j) amax = fmaxf(amax, fabsf(f[j]));
    }
  } else {
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) amax = fmaxf(amax, fabsf(to_f32<T>(row[i])));
  }
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  amax = 0.f;
  for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) amax = fmaxf(amax, red[i]);
  __syncthreads();  // red is reused by the caller
  return amax;
}

// One CTA per row: row_amax[r] = max_k |x[r, k]|.
template <typename T>
__global__ void __launch_bounds__(256) row_absmax_kernel(const T* __restrict__ x, int64_t k,
                                                         float* __restrict__ row_amax) {
  __shared__ float red[8];
  grid_launch_dependents();  // first kernel of a call: as split_activations_kernel
  grid_dependency_wait();
  const float a = row_absmax(x + static_cast<int64_t>(blockIdx.x) * k, k, red);
  if (threadIdx.x == 0) row_amax[blockIdx.x] = a;
}

// One CTA per row: s = amax / 448 with amax over the tensor (row_amax of every row, from
// row_absmax_kernel, which this grid may overlap until griddepcontrol.wait) or over the
// row; q[r, :] = e4m3(x[r, :] / s) and scale[r] = s.
template <typename T, bool kPerTensor>
__global__ void __launch_bounds__(256) quantize_dynamic_kernel(const T* __restrict__ x, int64_t rows, int64_t k,
                                                               const float* __restrict__ row_amax,
                                                               uint8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float red[8];
  // per tensor: second kernel, its primary is row_absmax_kernel; per row: the call's first
  // kernel, which (as split_activations_kernel) lets the GEMM launch before it waits for the
  // previous grid and reads x
  grid_launch_dependents();
  if (!kPerTensor) grid_dependency_wait();
  const int64_t r = blockIdx.x;
  const T* row = x + r * k;
  float amax = 0.f;
  if (kPerTensor) {
    grid_dependency_wait();
    for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) amax = fmaxf(amax, __ldcg(row_amax + i));
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.f;
    for (int i = 0; i < static_cast<int>(blockDim.x / 32); ++i) amax = fmaxf(amax, red[i]);
  } else {
    amax = row_absmax(row, k, red);
  }
  float s = __fdiv_rn(amax, 448.f);
  if (!(s > 0.f)) s = 1.f;
  uint8_t* qrow = q + r * k;
  constexpr int E = 16 / sizeof(T);
  if (row_vectorizable(row, k) && (reinterpret_cast<uintptr_t>(qrow) % E) == 0) {
    const uint4* v = reinterpret_cast<const uint4*>(row);
    for (int64_t i = threadIdx.x; i < k / E; i += blockDim.x) {
      float f[E];
      unpack16<T>(__ldg(v + i), f);
      uint8_t c[E];
#pragma unroll
      for (int j = 0; j < E; ++j) c[j] = to_e4m3(__fdiv_rn(f[j], s));
      if constexpr (E == 8) {
        uint2 o;
        o.x = c[0] | (c[1] << 8) | (c[2] << 16) | (static_cast<uint32_t>(c[3]) << 24);
        o.y = c[4] | (c[5] << 8) | (c[6] << 16) | (static_cast<uint32_t>(c[7]) << 24);
        *reinterpret_cast<uint2*>(qrow + i * E) = o;
      } else {
#pragma unroll
        for (int j = 0; j < E; ++j) qrow[i * E + j] = c[j];
      }
    }
  } else {
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) qrow[i] = to_e4m3(__fdiv_rn(to_f32<T>(row[i]), s));
  }
  if (threadIdx.x == 0) scale[r] = s;
}

// ---------------------------------------------------------------- weight packing
// packed[(nt * KT + kt) * 16384 + r * 128 + ((c16 ^ (r & 7)) * 16) + b] =
//     q[nt * 128 + r, kt * 128 + c16 * 16 + b]   (zero outside [N, K])
__global__ void __launch_bounds__(256) pack_weights_kernel(const uint8_t* __restrict__ q, int64_t n, int64_t k,
                                                           int64_t kt_count, uint4* __restrict__ packed,
                                                           int64_t chunks) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < chunks; i += step) {
    const int64_t tile = i >> 10;               // 1024 chunks of 16 B per tile
    const int within = static_cast<int>(i & 1023);
    const int r = within >> 3, cpos = within & 7;
    const int c16 = cpos ^ (r & 7);             // logical 16-byte chunk stored at cpos
    const int64_t nt = tile / kt_count, kt = tile - nt * kt_count;
    const int64_t row = nt * kTileN + r;
    const int64_t col = kt * kTileK + c16 * 16;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < n && col < k) {
      const uint8_t* src = q + row * k + col;
      if (col + 16 <= k && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        v = *reinterpret_cast<const uint4*>(src);
      } else {
        __align__(16) uint8_t tmp[16];
        for (int b = 0; b < 16; ++b) tmp[b] = (col + b < k) ? src[b] : 0;
        v = *reinterpret_cast<const uint4*>(tmp);
      }
    }
    packed[i] = v;
  }
}

// ---------------------------------------------------------------- host side
// Launch with programmatic stream serialisation: the grid may start while the previous
// one on the stream still runs; it calls griddepcontrol.wait before reading its output.
template <typename... KArgs, typename... Args>
inline int launch_pdl(dim3 grid, dim3 block, cudaStream_t s, void (*kernel)(KArgs...), Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

// 2-D tensor map over a row-major [rows, cols] array of 1-byte (u8) or 2-byte (bf16)
// elements with a (box_cols x box_rows) box; 128-byte swizzle optional.
struct MapKey {
  const void* base;
  uint64_t rows, cols;
  uint32_t box_cols, box_rows;
  int elem_bytes;
  bool swizzle;
  int dev;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && box_cols == o.box_cols &&
           box_rows == o.box_rows && elem_bytes == o.elem_bytes && swizzle == o.swizzle && dev == o.dev;
  }
};

inline int encode_map(CUtensorMap* map, const MapKey& k) {
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return INFERD_ERR_CUDA;
  cuuint64_t dims[2] = {k.cols, k.rows};
  cuuint64_t strides[1] = {k.cols * static_cast<uint64_t>(k.elem_bytes)};
  cuuint32_t box[2] = {k.box_cols, k.box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, k.elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                         const_cast<void*>(k.base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         k.swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? INFERD_OK : INFERD_ERR_CUDA;
}

// Small cache of encoded tensor maps: encoding costs microseconds of host time per map.
struct MapCache {
  std::mutex mu;
  struct Entry {
    MapKey key;
    CUtensorMap map;
  } e[48];
  int n = 0, next = 0;
};
MapCache g_maps;

inline int cached_map(CUtensorMap* map, const MapKey& key) {
  {
    std::lock_guard<std::mutex> lock(g_maps.mu);
    for (int i = 0; i < g_maps.n; ++i) {
      if (g_maps.e[i].key == key) {
        *map = g_maps.e[i].map;
        return INFERD_OK;
      }
    }
  }
  const int st = encode_map(map, key);
  if (st != INFERD_OK) return st;
  std::lock_guard<std::mutex> lock(g_maps.mu);
  g_maps.e[g_maps.next].key = key;
  g_maps.e[g_maps.next].map = *map;
  g_maps.next = (g_maps.next + 1) % 48;
  if (g_maps.n < 48) ++g_maps.n;
  return INFERD_OK;
}

// e4m3 planes and weights: 128-byte rows per box row
inline int cached_u8_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                         bool swizzle = true) {
  return cached_map(map, MapKey{base, rows, cols, static_cast<uint32_t>(kTileK), box_rows, 1, swizzle,
                                current_device()});
}

inline size_t align256_fp8(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// Workspace: [tile tickets: fixed region][h plane][l plane][x scales][partials].  The
// ticket region has one size for every call, so calls of any shape can share a
// workspace; completed calls leave the tickets at zero.  The dynamic-scaling calls use
// the l region for the per-row absmax; the partials region fits the plans of both kinds
// of call, so one workspace serves both.
constexpr int kMaxTilesFp8 = 4096;  // N <= 524288
constexpr size_t kFp8CounterBytes = kMaxTilesFp8 * sizeof(int32_t);

struct Fp8Plan {
  int tile;      // tokens per launch tile (multiple of 16)
  int stages;    // ring depth
  int per_sm;    // co-resident CTAs per SM
  int clusters;  // CTA pairs; the grid is 2 * clusters
  size_t smem;   // dynamic shared memory per CTA
};

// Weight-tile pairs of an [n, k] weight.
inline int64_t fp8_pairs(int64_t n) { return ((n + kTileN - 1) / kTileN + 1) / 2; }

inline Fp8Plan fp8_plan(int64_t rem_tokens, int64_t n, int64_t k, int sms, int planes) {
  Fp8Plan pl;
  const int64_t t = rem_tokens < kMaxTokTile ? rem_tokens : kMaxTokTile;
  pl.tile = static_cast<int>((t + 15) / 16 * 16);
  const int stage_bytes = kTileN * kTileK + fp8_x_stage_bytes(pl.tile, planes);
  const int64_t pairs = fp8_pairs(n);
  const int64_t work = pairs * ((k + kTileK - 1) / kTileK);
  const int64_t c1 = sms / 2;  // clusters at one CTA per SM
  if (pairs <= c1 && 4 * pairs >= 3 * c1) {
    // Whole tile pairs, one per cluster, one CTA per SM with the deepest ring: no partials
    // to merge and the most loads in flight per CTA (measured faster than two stream-K
    // CTAs per SM at every token count) -- used when the pairs keep three quarters of the
    // SM pairs busy.
    pl.per_sm = 1;
    pl.clusters = static_cast<int>(pairs);
  } else {
    // stream-K: two CTAs per SM while both double-buffered accumulators fit TMEM's 512
    // columns, at least four K steps per cluster
    pl.per_sm = 2 * fp8_tmem_cols(pl.tile, planes) <= 512 ? 2 : 1;
    int64_t c = c1 * pl.per_sm;
    const int64_t cap = work / 4 > 0 ? work / 4 : 1;
    if (c > cap) c = cap;
    // whole tile pairs at two CTAs per SM when they keep three quarters of those busy
    if (pairs <= c && 4 * pairs >= 3 * c) c = pairs;
    pl.clusters = static_cast<int>(c);
  }
  const int budget = pl.per_sm == 2 ? kSmemBudget2 : kSmemBudget;
  pl.stages = (budget - kEpiStageBytes) / stage_bytes;
  if (pl.stages > 8) pl.stages = 8;
  pl.smem = 1024 + static_cast<size_t>(pl.stages) * stage_bytes + kEpiStageBytes;
  return pl;
}

struct Fp8Workspace {
  size_t counters, h, l, scale, part, total;
};
inline Fp8Workspace fp8_workspace(int64_t m, int64_t n, int64_t k, int sms) {
  Fp8Workspace w;
  w.counters = 0;
  w.h = kFp8CounterBytes;
  w.l = w.h + align256_fp8(static_cast<size_t>(m * k));
  w.scale = w.l + align256_fp8(static_cast<size_t>(m * k));
  w.part = w.scale + align256_fp8(static_cast<size_t>(m) * 4);
  size_t part = 0;
  for (int planes = 1; planes <= 2; ++planes) {
    const Fp8Plan pl = fp8_plan(m, n, k, sms, planes);  // the first launch tile is the largest
    const size_t b = static_cast<size_t>(2 * (pl.clusters + fp8_pairs(n))) * pl.tile * kTileN * 4;
    if (b > part) part = b;
  }
  w.total = w.part + align256_fp8(part);
  return w;
}

}  // namespace
}  // namespace inferd

using namespace inferd;

inline int sm_count_of(int32_t device) {
  int sms = 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    sms = 148;
  }
  return sms;
}

extern "C" size_t inferd_fp8_linear_workspace_bytes(int64_t m, int64_t n, int64_t k, int32_t device) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return fp8_workspace(m, n, k, sm_count_of(device)).total;
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

extern "C" size_t inferd_fp8_packed_weight_bytes(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0) return 0;
  const int64_t nt = 2 * fp8_pairs(n), kt = (k + kTileK - 1) / kTileK;  // whole tile pairs
  return static_cast<size_t>(nt * kt) * kTileN * kTileK;
}

extern "C" int inferd_fp8_pack_weights(const void* w_e4m3, void* w_packed, int64_t n, int64_t k, void* stream) {
  if (n <= 0 || k <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (!w_e4m3 || !w_packed || (reinterpret_cast<uintptr_t>(w_packed) & 15) != 0)
    return INFERD_ERR_INVALID_ARGUMENT;
  const int64_t kt = (k + kTileK - 1) / kTileK;
  const int64_t chunks = static_cast<int64_t>(inferd_fp8_packed_weight_bytes(n, k)) / 16;
  int64_t blocks = (chunks + 255) / 256;
  const int64_t cap = static_cast<int64_t>(current_sm_count()) * 32;
  if (blocks > cap) blocks = cap;
  pack_weights_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(w_e4m3), n, k, kt, static_cast<uint4*>(w_packed), chunks);
  return launch_status();
}

// Activation preparation of one call: 0 = exact two-plane split (weight-only FP8),
// 1 = one e4m3 plane scaled by the tensor's absmax, 2 = one plane scaled per row.
enum Fp8ActMode { kActSplit = 0, kActDynTensor = 1, kActDynRow = 2 };

static int fp8_linear_impl(void* y, const void* x, const void* w_e4m3, const float* w_scale, int64_t m, int64_t n,
                           int64_t k, int32_t w_layout, int act_mode, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (w_layout != 0 && w_layout != 1) return INFERD_ERR_INVALID_ARGUMENT;
  if (m < 0 || n <= 0 || k <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (m == 0) return INFERD_OK;
  if (!y || !x || !w_e4m3 || !w_scale) return INFERD_ERR_INVALID_ARGUMENT;
  if (k % 16 != 0) return INFERD_ERR_UNSUPPORTED;  // TMA rows must be 16-byte multiples
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff) return INFERD_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(w_e4m3) & 15) != 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
    return INFERD_ERR_INVALID_ARGUMENT;  // 16-byte aligned weights and activations
  if ((n + kTileN - 1) / kTileN > kMaxTilesFp8) return INFERD_ERR_UNSUPPORTED;
  const int planes = act_mode == kActSplit ? 2 : 1;
  const int sms = current_sm_count();
  const Fp8Workspace wl = fp8_workspace(m, n, k, sms);
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0 || workspace_bytes < wl.total)
    return INFERD_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint8_t* h = ws + wl.h;
  uint8_t* l = ws + wl.l;
  float* xs = reinterpret_cast<float*>(ws + wl.scale);
  int32_t* counters = reinterpret_cast<int32_t*>(ws + wl.counters);
  float* part = reinterpret_cast<float*>(ws + wl.part);

  static bool configured[64] = {false};
  const int dev = current_device();
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(fp8_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 1024);
    if (e != cudaSuccess) return cuda_status(e);
    // all of the unified L1/shared array as shared memory, so two ~110 KB CTAs fit per SM;
    // the activation kernels ask for the same carveout, so the SMs are not reconfigured
    // between the launches of a call
    const void* kernels[] = {reinterpret_cast<const void*>(fp8_linear_kernel),
                             reinterpret_cast<const void*>(split_activations_kernel),
                             reinterpret_cast<const void*>(row_absmax_kernel<__nv_bfloat16>),
                             reinterpret_cast<const void*>(quantize_dynamic_kernel<__nv_bfloat16, true>),
                             reinterpret_cast<const void*>(quantize_dynamic_kernel<__nv_bfloat16, false>)};
    for (const void* f : kernels) {
      e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return cuda_status(e);
    }
    configured[dev] = true;
  }

  // encode every tensor map before the first launch so no host work separates the
  // kernels of a call
  const int n_tok_tiles = static_cast<int>((m + kMaxTokTile - 1) / kMaxTokTile);
  CUtensorMap wmap;
  int st = INFERD_OK;
  if (w_layout == 0) {
    st = cached_u8_map(&wmap, w_e4m3, static_cast<uint64_t>(n), static_cast<uint64_t>(k), kTileN);
  } else {
    // packed tiles are already in shared-memory form: copy them verbatim as 128-byte rows
    const uint64_t rows = static_cast<uint64_t>(inferd_fp8_packed_weight_bytes(n, k)) / kTileK;
    st = cached_u8_map(&wmap, w_e4m3, rows, kTileK, kTileN, false);
  }
  if (st != INFERD_OK) return st;
  // y through TMA stores when its rows are 16-byte multiples at a 16-byte aligned base
  CUtensorMap ymap;
  const bool y_tma = (n * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  if (y_tma) {
    st = cached_map(&ymap, MapKey{y, static_cast<uint64_t>(m), static_cast<uint64_t>(n), 32, 32, 2, false,
                                  current_device()});
    if (st != INFERD_OK) return st;
  } else {
    memset(&ymap, 0, sizeof(ymap));
  }
  CUtensorMap hmaps[2], lmaps[2];  // full tiles share one map; a last partial tile its own
  int tiles[2];
  for (int i = 0; i < 2; ++i) {
    const int64_t rem =
        i == 0 ? (m < kMaxTokTile ? m : kMaxTokTile) : m - static_cast<int64_t>(n_tok_tiles - 1) * kMaxTokTile;
    tiles[i] = static_cast<int>((rem + 15) / 16 * 16);
    // rows each CTA of the pair loads per plane: the whole tile (two planes, tile <= 128)
    // or half of it
    const uint32_t box = static_cast<uint32_t>(planes == 2 && tiles[i] <= 128 ? tiles[i] : tiles[i] / 2);
    st = cached_u8_map(&hmaps[i], h, static_cast<uint64_t>(m), static_cast<uint64_t>(k), box);
    if (st != INFERD_OK) return st;
    if (planes == 2) {
      st = cached_u8_map(&lmaps[i], l, static_cast<uint64_t>(m), static_cast<uint64_t>(k), box);
      if (st != INFERD_OK) return st;
    } else {
      lmaps[i] = hmaps[i];  // not read
    }
  }

  const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(x);
  // every kernel of the call is a programmatic dependent launch; see the kernels' waits
  if (act_mode == kActSplit) {
    st = launch_pdl(dim3(static_cast<unsigned>(m)), dim3(kSplitThreads), s, split_activations_kernel, xb,
                    static_cast<int>(k), h, l, xs);
  } else if (act_mode == kActDynRow) {
    st = launch_pdl(dim3(static_cast<unsigned>(m)), dim3(256), s, quantize_dynamic_kernel<__nv_bfloat16, false>, xb,
                    m, k, static_cast<const float*>(nullptr), h, xs);
  } else {
    float* row_amax = reinterpret_cast<float*>(l);
    st = launch_pdl(dim3(static_cast<unsigned>(m)), dim3(256), s, row_absmax_kernel<__nv_bfloat16>, xb, k, row_amax);
    if (st != INFERD_OK) return st;
    st = launch_pdl(dim3(static_cast<unsigned>(m)), dim3(256), s, quantize_dynamic_kernel<__nv_bfloat16, true>, xb,
                    m, k, static_cast<const float*>(row_amax), h, xs);
  }
  if (st == INFERD_OK) st = launch_status();
  if (st != INFERD_OK) return st;

  for (int t = 0; t < n_tok_tiles; ++t) {
    const int which = (t == n_tok_tiles - 1) ? 1 : 0;
    const Fp8Plan pl = fp8_plan(m - static_cast<int64_t>(t) * kMaxTokTile, n, k, sms, planes);
    const int tile = tiles[which];
    if (pl.stages < 2 || pl.tile != tile) return INFERD_ERR_UNSUPPORTED;
    // The cluster-occupancy query reports one cluster per SM pair for the two-per-SM
    // configurations, yet launching two per pair measures faster; stream-K needs no
    // co-residency, so the grid is not clamped to it.
    const int clusters = pl.clusters;
    Fp8Params p;
    p.y = static_cast<__nv_bfloat16*>(y);
    p.w_scale = w_scale;
    p.x_scale = xs;
    p.m = static_cast<int32_t>(m);
    p.n = static_cast<int32_t>(n);
    p.k = static_cast<int32_t>(k);
    p.w_packed = w_layout == 1 ? 1 : 0;
    p.tok0 = t * kMaxTokTile;
    p.tok_tile = tile;
    p.stages = pl.stages;
    p.counters = counters;
    p.part = part;
    p.error_word = nullptr;
    p.y_tma = y_tma ? 1 : 0;
    p.planes = planes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(kFp8Threads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    st = cuda_status(cudaLaunchKernelEx(&cfg, fp8_linear_kernel, wmap, hmaps[which], lmaps[which], ymap, p));
    if (st != INFERD_OK) return st;
  }
  return INFERD_OK;
}

extern "C" int inferd_fp8_linear(void* y, const void* x, const void* w_e4m3, const float* w_scale, int64_t m,
                                 int64_t n, int64_t k, int32_t w_layout, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  return fp8_linear_impl(y, x, w_e4m3, w_scale, m, n, k, w_layout, kActSplit, workspace, workspace_bytes, stream);
}

extern "C" int inferd_fp8_dynamic_linear(void* y, const void* x, const void* w_e4m3, const float* w_scale,
                                         int64_t m, int64_t n, int64_t k, int32_t w_layout, int32_t granularity,
                                         void* workspace, size_t workspace_bytes, void* stream) {
  if (granularity != INFERD_FP8_PER_TENSOR && granularity != INFERD_FP8_PER_ROW) return INFERD_ERR_INVALID_ARGUMENT;
  return fp8_linear_impl(y, x, w_e4m3, w_scale, m, n, k, w_layout,
                         granularity == INFERD_FP8_PER_TENSOR ? kActDynTensor : kActDynRow, workspace,
                         workspace_bytes, stream);
}

template <typename T>
static int quantize_dynamic_launch(const T* x, int64_t rows, int64_t k, int32_t granularity, uint8_t* q,
                                   float* scale, float* row_amax, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(rows));
  if (granularity == INFERD_FP8_PER_ROW) {
    quantize_dynamic_kernel<T, false><<<grid, 256, 0, s>>>(x, rows, k, nullptr, q, scale);
    return launch_status();
  }
  row_absmax_kernel<T><<<grid, 256, 0, s>>>(x, k, row_amax);
  const int st = launch_status();
  if (st != INFERD_OK) return st;
  return launch_pdl(grid, dim3(256), s, quantize_dynamic_kernel<T, true>, x, rows, k,
                    static_cast<const float*>(row_amax), q, scale);
}

extern "C" int inferd_fp8_quantize_dynamic(const void* x, int32_t x_dtype, void* q, float* scale, int64_t rows,
                                           int64_t k, int32_t granularity, float* row_amax, void* stream) {
  if (rows < 0 || k <= 0) return INFERD_ERR_INVALID_ARGUMENT;
  if (granularity != INFERD_FP8_PER_TENSOR && granularity != INFERD_FP8_PER_ROW) return INFERD_ERR_INVALID_ARGUMENT;
  if (rows == 0) return INFERD_OK;
  if (!x || !q || !scale || (granularity == INFERD_FP8_PER_TENSOR && !row_amax)) return INFERD_ERR_INVALID_ARGUMENT;
  if (rows > 0x7fffffff) return INFERD_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* qb = static_cast<uint8_t*>(q);
  if (x_dtype == INFERD_BF16)
    return quantize_dynamic_launch(static_cast<const __nv_bfloat16*>(x), rows, k, granularity, qb, scale, row_amax, s);
  if (x_dtype == INFERD_F16)
    return quantize_dynamic_launch(static_cast<const __half*>(x), rows, k, granularity, qb, scale, row_amax, s);
  if (x_dtype == INFERD_F32)
    return quantize_dynamic_launch(static_cast<const float*>(x), rows, k, granularity, qb, scale, row_amax, s);
  return INFERD_ERR_UNSUPPORTED;
}
