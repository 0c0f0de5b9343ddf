// cache_ops.cu -- KV-pool writes (reshape_and_cache) and page gathers.
//
// Both are pure byte movement, bound by HBM bandwidth: every (token, kv-head) row of
// head_dim elements is moved in 16-byte units whenever the row size, base pointers and
// strides allow it, so a warp moves 512 contiguous bytes per instruction.
#include "common.cuh"
#include "runtime.cuh"

namespace inferd {
namespace {

// One thread moves one copy unit U of one (token, head) row of K and the same unit of V.
// Replaces core/paged_cache.py:177-183: for each new token, (page, offset) =
// divmod(pos, block_size) and key_cache[block, :, offset, :] = keys[token].  The slot
// (block * block_size + offset) is computed on the host from the page table.
template <typename U>
__global__ void __launch_bounds__(256) reshape_and_cache_kernel(
    const uint8_t* __restrict__ key, const uint8_t* __restrict__ value, int64_t kts, int64_t khs,
    int64_t vts, int64_t vhs, U* __restrict__ key_cache, U* __restrict__ value_cache,
    const int64_t* __restrict__ slots, int64_t num_tokens, int32_t num_kv_heads, int32_t row_units,
    int32_t block_size, int64_t num_blocks, int32_t* error_word) {
  const int64_t total = num_tokens * num_kv_heads * row_units;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += step) {
    const int64_t u = i % row_units;
    const int64_t th = i / row_units;
    const int64_t h = th % num_kv_heads;
    const int64_t t = th / num_kv_heads;
    const int64_t slot = __ldg(slots + t);
    if (slot < 0) continue;  // padding token: nothing to write
    const int64_t blk = slot / block_size;
    const int64_t off = slot - blk * block_size;
    if (blk >= num_blocks) {
      report_error(error_word, INFERD_ERR_DEVICE_INDEX);
      continue;
    }
    const int64_t dst = ((blk * num_kv_heads + h) * block_size + off) * row_units + u;
    const U kv = *reinterpret_cast<const U*>(key + t * kts + h * khs + u * sizeof(U));
    const U vv = *reinterpret_cast<const U*>(value + t * vts + h * vhs + u * sizeof(U));
    key_cache[dst] = kv;
    value_cache[dst] = vv;
  }
}

// out[t, h, :] = cache[table[t / bs], h, t % bs, :] for t < seq_len.
// Replaces core/paged_attn.py:48-61 (per-page slice + transpose + cat) and
// core/paged_cache.py:201-204 (per-position copy).
template <typename U, typename Idx>
__global__ void __launch_bounds__(256) gather_kernel(
    U* __restrict__ key_out, U* __restrict__ value_out, const U* __restrict__ key_cache,
    const U* __restrict__ value_cache, const Idx* __restrict__ table, int64_t seq_len,
    int32_t num_kv_heads, int32_t row_units, int32_t block_size, int64_t num_blocks,
    int32_t* error_word) {
  const int64_t total = seq_len * num_kv_heads * row_units;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += step) {
    const int64_t u = i % row_units;
    const int64_t th = i / row_units;
    const int64_t h = th % num_kv_heads;
    const int64_t t = th / num_kv_heads;
    const int64_t page = t / block_size;
    const int64_t off = t - page * block_size;
    const int64_t blk = static_cast<int64_t>(__ldg(table + page));
    U kv, vv;
    if (blk < 0 || blk >= num_blocks) {
      report_error(error_word, INFERD_ERR_DEVICE_INDEX);
      kv = U{};
      vv = U{};
    } else {
      const int64_t src = ((blk * num_kv_heads + h) * block_size + off) * row_units + u;
      kv = key_cache[src];
      vv = value_cache[src];
    }
    key_out[i] = kv;
    value_out[i] = vv;
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline unsigned grid_for(int64_t total) {
  const int64_t want = (total + 255) / 256;
  const int64_t cap = static_cast<int64_t>(current_sm_count()) * 16;
  return static_cast<unsigned>(want < 1 ? 1 : (want > cap ? cap : want));
}

template <typename U>
int launch_reshape(const void* key, const void* value, int64_t kts, int64_t khs, int64_t vts,
                   int64_t vhs, void* kc, void* vc, const int64_t* slots, int64_t n, int32_t hkv,
                   int32_t row_bytes, int32_t bs, int64_t nb, int32_t* err, cudaStream_t s) {
  const int32_t units = row_bytes / static_cast<int32_t>(sizeof(U));
  const int64_t total = n * hkv * units;
  reshape_and_cache_kernel<U><<<grid_for(total), 256, 0, s>>>(
      static_cast<const uint8_t*>(key), static_cast<const uint8_t*>(value), kts, khs, vts, vhs,
      static_cast<U*>(kc), static_cast<U*>(vc), slots, n, hkv, units, bs, nb, err);
  return launch_status();
}

template <typename U, typename Idx>
int launch_gather(void* ko, void* vo, const void* kc, const void* vc, const void* table,
                  int64_t len, int32_t hkv, int32_t row_bytes, int32_t bs, int64_t nb,
                  int32_t* err, cudaStream_t s) {
  const int32_t units = row_bytes / static_cast<int32_t>(sizeof(U));
  const int64_t total = len * hkv * units;
  gather_kernel<U, Idx><<<grid_for(total), 256, 0, s>>>(
      static_cast<U*>(ko), static_cast<U*>(vo), static_cast<const U*>(kc),
      static_cast<const U*>(vc), static_cast<const Idx*>(table), len, hkv, units, bs, nb, err);
  return launch_status();
}

// Packed decode metadata kept on the device across steps.  Block r updates row r of the
// master table [rows, capacity] -- dense: the whole row from src (a [rows, capacity] upload);
// sparse: the entries src[row_ptr[r] .. row_ptr[r+1]) = (column, block) pairs -- and then
// copies its first `width` entries to out [rows, width].  Rows are independent, so one
// launch both applies the step's page-table changes and produces the table the attention
// kernels read.
__global__ void __launch_bounds__(256) block_tables_refresh_kernel(int32_t* __restrict__ master, int64_t cap,
                                                                   const int32_t* __restrict__ row_ptr,
                                                                   const int32_t* __restrict__ src, int32_t dense,
                                                                   int32_t width, int32_t* __restrict__ out) {
  const int64_t r = blockIdx.x;
  int32_t* row = master + r * cap;
  if (dense) {
    for (int64_t c = threadIdx.x; c < cap; c += blockDim.x) row[c] = __ldg(src + r * cap + c);
  } else {
    const int32_t e0 = __ldg(row_ptr + r), e1 = __ldg(row_ptr + r + 1);
    for (int32_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
      const int32_t col = __ldg(src + 2 * e), blk = __ldg(src + 2 * e + 1);
      if (col >= 0 && col < cap) row[col] = blk;
    }
  }
  __syncthreads();
  for (int64_t c = threadIdx.x; c < width; c += blockDim.x) out[r * width + c] = row[c];
}

}  // namespace
}  // namespace inferd

using namespace inferd;

extern "C" int inferd_block_tables_refresh(int32_t* master, int64_t capacity, const int32_t* row_ptr,
                                           const int32_t* updates, int32_t dense, int32_t num_rows,
                                           int32_t width, int32_t* block_tables, void* stream) {
  if (num_rows < 0 || capacity <= 0 || width < 0 || width > capacity) return INFERD_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return INFERD_OK;
  if (!master || !updates || !block_tables || (!dense && !row_ptr)) return INFERD_ERR_INVALID_ARGUMENT;
  block_tables_refresh_kernel<<<static_cast<unsigned>(num_rows), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      master, capacity, row_ptr, updates, dense ? 1 : 0, width, block_tables);
  return launch_status();
}

extern "C" int inferd_reshape_and_cache(const void* key, const void* value,
                                        int64_t key_token_stride, int64_t key_head_stride,
                                        int64_t value_token_stride, int64_t value_head_stride,
                                        void* key_cache, void* value_cache,
                                        const int64_t* slot_mapping, int64_t num_tokens,
                                        int32_t num_kv_heads, int32_t head_dim,
                                        int32_t block_size, int64_t num_blocks, int32_t dtype,
                                        int32_t* error_word, void* stream) {
  if (num_tokens < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0)
    return INFERD_ERR_INVALID_ARGUMENT;
  if (dtype < INFERD_F32 || dtype > INFERD_E4M3) return INFERD_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return INFERD_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping)
    return INFERD_ERR_INVALID_ARGUMENT;
  const int64_t es = dtype_bytes(dtype);
  const int32_t row_bytes = static_cast<int32_t>(head_dim * es);
  const int64_t kts = key_token_stride * es, khs = key_head_stride * es;
  const int64_t vts = value_token_stride * es, vhs = value_head_stride * es;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec16 = (row_bytes % 16 == 0) && aligned16(key) && aligned16(value) &&
                     aligned16(key_cache) && aligned16(value_cache) && kts % 16 == 0 &&
                     khs % 16 == 0 && vts % 16 == 0 && vhs % 16 == 0;
  if (vec16)
    return launch_reshape<uint4>(key, value, kts, khs, vts, vhs, key_cache, value_cache,
                                 slot_mapping, num_tokens, num_kv_heads, row_bytes, block_size,
                                 num_blocks, error_word, s);
  if (es == 4)
    return launch_reshape<uint32_t>(key, value, kts, khs, vts, vhs, key_cache, value_cache,
                                    slot_mapping, num_tokens, num_kv_heads, row_bytes, block_size,
                                    num_blocks, error_word, s);
  if (es == 2)
    return launch_reshape<uint16_t>(key, value, kts, khs, vts, vhs, key_cache, value_cache,
                                    slot_mapping, num_tokens, num_kv_heads, row_bytes, block_size,
                                    num_blocks, error_word, s);
  return launch_reshape<uint8_t>(key, value, kts, khs, vts, vhs, key_cache, value_cache,
                                 slot_mapping, num_tokens, num_kv_heads, row_bytes, block_size,
                                 num_blocks, error_word, s);
}

extern "C" int inferd_gather_paged_kv(void* key_out, void* value_out, const void* key_cache,
                                      const void* value_cache, const void* block_table,
                                      int32_t block_table_bytes, int64_t seq_len,
                                      int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                      int64_t num_blocks, int32_t dtype, int32_t* error_word,
                                      void* stream) {
  if (seq_len < 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || num_blocks <= 0)
    return INFERD_ERR_INVALID_ARGUMENT;
  if (block_table_bytes != 4 && block_table_bytes != 8) return INFERD_ERR_INVALID_ARGUMENT;
  if (dtype < INFERD_F32 || dtype > INFERD_E4M3) return INFERD_ERR_INVALID_ARGUMENT;
  if (seq_len == 0) return INFERD_OK;
  if (!key_out || !value_out || !key_cache || !value_cache || !block_table)
    return INFERD_ERR_INVALID_ARGUMENT;
  const int32_t es = dtype_bytes(dtype);
  const int32_t row_bytes = head_dim * es;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec16 = (row_bytes % 16 == 0) && aligned16(key_out) && aligned16(value_out) &&
                     aligned16(key_cache) && aligned16(value_cache);
  const bool i64 = block_table_bytes == 8;
#define INFERD_GATHER(U)                                                                      \
  (i64 ? launch_gather<U, int64_t>(key_out, value_out, key_cache, value_cache, block_table,   \
                                   seq_len, num_kv_heads, row_bytes, block_size, num_blocks,  \
                                   error_word, s)                                             \
       : launch_gather<U, int32_t>(key_out, value_out, key_cache, value_cache, block_table,   \
                                   seq_len, num_kv_heads, row_bytes, block_size, num_blocks,  \
                                   error_word, s))
  if (vec16) return INFERD_GATHER(uint4);
  if (es == 4) return INFERD_GATHER(uint32_t);
  if (es == 2) return INFERD_GATHER(uint16_t);
  return INFERD_GATHER(uint8_t);
#undef INFERD_GATHER
}
