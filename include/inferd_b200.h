/*
 * inferd_b200.h -- C ABI of the sm_100a decode hot path (libinferd_sm100a.so).
 *
 * Every entry point takes raw device pointers, sizes and a cudaStream_t passed as
 * `void*`, enqueues its kernels on that stream and returns an `int` status from
 * inferd_status_t without synchronising.  No torch or CUDA types appear in the
 * signatures, so the library can be bound from ctypes, cgo, JNI or N-API alike.
 *
 * Tensor layouts (all contiguous in the innermost dimension):
 *   KV pool      key_cache / value_cache : [num_blocks, num_kv_heads, block_size, head_dim]
 *                (core/paged_cache.py:131-137 of the reference)
 *   query / out  [num_seqs, q_len, num_q_heads, head_dim]
 *   block table  [num_seqs, block_table_stride] of int32 or int64 block ids
 *   slot mapping [num_tokens] int64, slot = block * block_size + offset; slot < 0 skips
 *
 * Device-detected errors (a block id or slot outside the pool, a bounded wait that
 * expired) never trap: the kernel records the first error code in *error_word
 * (when error_word is non-NULL), skips or clamps the offending access and finishes.
 * The caller reads the word whenever it chooses to synchronise.
 */
#ifndef INFERD_B200_H
#define INFERD_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define INFERD_API __attribute__((visibility("default")))
#else
#define INFERD_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  INFERD_OK = 0,
  INFERD_ERR_INVALID_ARGUMENT = 1, /* shape / argument error (Python: ValueError)          */
  INFERD_ERR_UNSUPPORTED = 2,      /* combination of dtype / sizes not built                 */
  INFERD_ERR_WORKSPACE = 3,        /* workspace missing, misaligned or too small             */
  INFERD_ERR_CUDA = 4,             /* launch or runtime failure                              */
  INFERD_ERR_DEVICE_INDEX = 5,     /* device side: block id / slot outside the pool (IndexError) */
  INFERD_ERR_DEVICE_TIMEOUT = 6    /* device side: a bounded wait expired                    */
} inferd_status_t;

typedef enum {
  INFERD_F32 = 0,
  INFERD_F16 = 1,
  INFERD_BF16 = 2,
  INFERD_E4M3 = 3
} inferd_dtype_t;

/* Library version (major * 10000 + minor * 100 + patch). */
INFERD_API int inferd_version(void);

/* Static description of a status code. */
INFERD_API const char* inferd_status_string(int status);

/* Last CUDA error string recorded by a failing call on this thread ("" if none). */
INFERD_API const char* inferd_last_cuda_error(void);

/*
 * Device address of page-locked host memory (cudaHostAlloc / cudaMallocHost), which
 * kernels may read and write directly; under unified addressing it equals the host
 * address.  INFERD_ERR_CUDA for pageable or unregistered memory.  A caller can hand it
 * to inferd_paged_attention_gather as a destination, so that the attention's epilogue
 * copies its output rows to the host while the grid still runs instead of a separate
 * device-to-host copy after it.  No counterpart in the reference.
 */
INFERD_API int inferd_host_device_pointer(const void* host, void** device_ptr);

/*
 * reshape_and_cache: write num_tokens new K/V rows into their pool slots.
 * Replaces the write loop of PagedKVCache.append_tokens, core/paged_cache.py:177-183
 * (key_cache[layer][block, :, offset, :] = layer_keys[layer][rel_pos]); the page-table
 * bookkeeping of :164-176,184-189 stays on the host.  key/value element (t, h, d) is at
 * key[t * key_token_stride + h * key_head_stride + d] (strides in elements).
 * Bit-exact copy for every dtype.
 */
INFERD_API int inferd_reshape_and_cache(const void* key, const void* value,
                             int64_t key_token_stride, int64_t key_head_stride,
                             int64_t value_token_stride, int64_t value_head_stride,
                             void* key_cache, void* value_cache,
                             const int64_t* slot_mapping, int64_t num_tokens,
                             int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                             int64_t num_blocks, int32_t dtype,
                             int32_t* error_word, void* stream);

/*
 * Device-resident decode metadata.  master [num_rows, capacity] int32 holds the batch's
 * page tables across steps; one call applies this step's changes and writes the packed
 * block_tables [num_rows, width] the attention kernels read.  dense = 1: updates is the whole
 * [num_rows, capacity] table (row_ptr unused); dense = 0: row r's changes are the
 * (column, block) int32 pairs updates[2 * row_ptr[r] .. 2 * row_ptr[r + 1]).  Replaces the
 * per-step block_table() rebuild and host->device copy of core/paged_cache.py:207-213.
 */
INFERD_API int inferd_block_tables_refresh(int32_t* master, int64_t capacity, const int32_t* row_ptr,
                                           const int32_t* updates, int32_t dense, int32_t num_rows,
                                           int32_t width, int32_t* block_tables, void* stream);

/*
 * gather_paged_kv: copy one sequence's pages back to contiguous [seq_len, num_kv_heads,
 * head_dim] tensors.  Replaces core/paged_attn.py:20-61 (gather_paged_kv) and
 * core/paged_cache.py:191-205 (PagedKVCache.gather_layer).  Bit-exact.
 * block_table_bytes is 4 (int32) or 8 (int64).
 */
INFERD_API int inferd_gather_paged_kv(void* key_out, void* value_out,
                           const void* key_cache, const void* value_cache,
                           const void* block_table, int32_t block_table_bytes,
                           int64_t seq_len, int32_t num_kv_heads, int32_t head_dim,
                           int32_t block_size, int64_t num_blocks, int32_t dtype,
                           int32_t* error_word, void* stream);

/*
 * Paged attention over the block-table pool, batched over sequences.
 *   q_len == 1 : decode attention, replaces core/paged_attn.py:147-167 paged_attention
 *                (-> paged_attention_reference :134-144 -> gather :20-61 + dense :64-106).
 *   q_len  > 1 : causal multi-query verify attention of speculative decoding, replacing the
 *                target verify forward core/spec_decode.py:135 (HF eager attention over
 *                contiguous KV).  Query i of sequence b sits at absolute position
 *                context_lens[b] - q_len + i and sees keys 0 .. that position; the q_len
 *                window's own K/V must already be in the pool (reshape_and_cache first).
 * GQA: query head hq reads kv head hq / (num_q_heads / num_kv_heads), the
 * repeat_interleave order of core/paged_attn.py:99-100.
 * context_lens: [num_seqs] int32 on the device, or NULL for "every sequence has
 * max_context_len keys".  max_context_len is a host-side upper bound used for grid sizing.
 * A sequence with no visible keys gets an all-zero output row (softmax over nothing).
 * workspace: >= inferd_paged_attention_workspace_bytes(...) bytes, 256-byte aligned.  It
 * starts with a fixed 512 KiB ticket-counter region (partials are stored after it, whatever
 * the call's shape); the first inferd_paged_attention_counter_bytes(num_seqs,
 * num_kv_heads) bytes of that region are used by a call, must be zero before it, and are
 * left zero by every completed call -- zero the region once when the workspace is
 * allocated and it can be shared by calls of any shape.  Calls that share a workspace
 * must be ordered on one stream.
 * A call with q_len * (num_q_heads / num_kv_heads) > 8 enqueues two kernels on `stream`:
 * the paged attention kernel, and a kernel that merges the sequences it split across
 * warps (launched with programmatic stream serialization; both are captured together by
 * a CUDA graph).
 */
INFERD_API int inferd_paged_attention(void* out, const void* query,
                           const void* key_cache, const void* value_cache,
                           const void* block_tables, int32_t block_table_bytes,
                           int64_t block_table_stride, const int32_t* context_lens,
                           int32_t num_seqs, int32_t q_len, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                           int64_t num_blocks, int32_t max_context_len, float scale,
                           int32_t dtype, void* workspace, size_t workspace_bytes,
                           int32_t* error_word, void* stream);

INFERD_API size_t inferd_paged_attention_workspace_bytes(int32_t num_seqs, int32_t q_len,
                                              int32_t num_q_heads, int32_t num_kv_heads,
                                              int32_t head_dim, int32_t device);

INFERD_API size_t inferd_paged_attention_counter_bytes(int32_t num_seqs, int32_t num_kv_heads);

/*
 * inferd_paged_attention without a caller-provided workspace: same arguments, results
 * and status codes as inferd_paged_attention minus (workspace, workspace_bytes).
 * No counterpart in the reference; it exists for callers that cannot allocate device
 * memory at call time (FFI hosts without a device allocator, serving loops whose device
 * memory budget is fixed at start-up).  It calls no cudaMalloc/cudaFree and no
 * allocating library routine.
 * Scratch: a 32 MiB static device array inside the library, held by every GPU that loads
 * the library until the process exits.  A call that runs on the tensor-core path and
 * needs more than that (inferd_paged_attention_workspace_bytes(...) > 32 MiB) returns
 * INFERD_ERR_WORKSPACE; calls on the generic path (fp32, head_dim != 128, block_size != 16,
 * more than 32 query rows per kv head) use no scratch and are not limited.
 * The first call on a device looks up the array's device address (once per device, with
 * that device current); make that first call before any stream capture.  The address is
 * kept for the life of the process and is not looked up again after cudaDeviceReset() or
 * another change of the device's primary context: do not call this entry point on that
 * device after one.  Every call clears the ticket counters itself; all calls share the
 * array, so calls that overlap on the GPU race -- order them on one stream.
 */
INFERD_API int inferd_paged_attention_noalloc(void* out, const void* query,
                           const void* key_cache, const void* value_cache,
                           const void* block_tables, int32_t block_table_bytes,
                           int64_t block_table_stride, const int32_t* context_lens,
                           int32_t num_seqs, int32_t q_len, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                           int64_t num_blocks, int32_t max_context_len, float scale,
                           int32_t dtype, int32_t* error_word, void* stream);

/*
 * Dense (contiguous) attention: query [q_len, num_q_heads, head_dim] against key/value
 * [seq_len, num_kv_heads, head_dim].  q_len == 1 is core/paged_attn.py:64-106
 * dense_attention (no mask); q_len > 1 applies the same causal rule as
 * inferd_paged_attention.  Accumulates in fp32.
 */
INFERD_API int inferd_dense_attention(void* out, const void* query, const void* key, const void* value,
                           int64_t seq_len, int32_t q_len, int32_t num_q_heads,
                           int32_t num_kv_heads, int32_t head_dim, float scale, int32_t dtype,
                           void* stream);

/*
 * Load-time FP8 weight quantisation, per output channel: s[n] = max_k |W[n, k]| / 448 in
 * fp32 (1 for an all-zero row) and w_e4m3[n, k] = e4m3(W[n, k] / s[n]), IEEE division,
 * round-to-nearest-even, saturating.  Replaces torchao 0.17.0 Float8WeightOnlyConfig as
 * configured in bench/model_loader.py:46-58 (applied at :82-88).  w_dtype: f32/f16/bf16.
 */
INFERD_API int inferd_fp8_quantize_per_channel(const void* w, int32_t w_dtype, void* w_e4m3,
                                               float* w_scale, int64_t n, int64_t k,
                                               void* stream);

/*
 * Load-time repacking of row-major e4m3 weights [N, K] into the tile layout the linear
 * streams fastest: every 128-row x 128-byte tile is one contiguous 16 KiB block (already
 * in the MMA's 128-byte-swizzled form), the tiles of a 128-row band consecutive along K,
 * zero-filled past N and K; the band count is rounded up to even (whole 256-row pairs).  w_packed needs inferd_fp8_packed_weight_bytes(n, k) bytes,
 * 16-byte aligned.  No counterpart in the reference (its torchao weights stay row-major).
 */
INFERD_API size_t inferd_fp8_packed_weight_bytes(int64_t n, int64_t k);
INFERD_API int inferd_fp8_pack_weights(const void* w_e4m3, void* w_packed, int64_t n, int64_t k,
                                       void* stream);

/*
 * y[m, n] = s[n] * sum_k x[m, k] * w[n, k]: x bf16 [M, K], w_scale fp32 [N], y bf16 [M, N],
 * row-major; K % 16 == 0.  w_layout 0: w_e4m3 row-major [N, K]; 1: packed by
 * inferd_fp8_pack_weights.  w must be 16-byte aligned.  The FP8 weight-only linear the
 * reference runs through torchao (bench/model_loader.py:46-58; caller
 * core/model_runner.py:27-45).  tcgen05 kind::f8f6f4 tensor cores with the activations
 * split exactly into two e4m3 planes under a power-of-two row scale.
 * workspace >= inferd_fp8_linear_workspace_bytes(m, n, k, device), 256-byte aligned.
 */
INFERD_API int inferd_fp8_linear(void* y, const void* x, const void* w_e4m3,
                                 const float* w_scale, int64_t m, int64_t n, int64_t k,
                                 int32_t w_layout, void* workspace, size_t workspace_bytes,
                                 void* stream);

INFERD_API size_t inferd_fp8_linear_workspace_bytes(int64_t m, int64_t n, int64_t k,
                                                    int32_t device);

/*
 * FP8 with dynamic activation scaling: the reference's "fp8-dynamic" recipe, torchao 0.17.0
 * Float8DynamicActivationFloat8WeightConfig() (bench/model_loader.py:53-55; granularity
 * PerTensor by default, PerRow optional).  A tensor (or row) is quantised as
 * s = amax / 448 in fp32 (1 when amax is 0), q = e4m3(x / s): IEEE division,
 * round-to-nearest-even, saturating at +-448 (torchao's clamp before the cast).
 *
 * inferd_fp8_quantize_dynamic: x [rows, k] (f32/f16/bf16) -> q e4m3 [rows, k] and
 * scale fp32 [rows] (per tensor: every entry holds the tensor's scale).  Per tensor needs
 * row_amax, rows floats of scratch; per row ignores it.  Used at load time for the weights
 * (every row of scale then feeds the linear's w_scale) and by the linear for activations.
 *
 * inferd_fp8_dynamic_linear: y[m, n] = s_x[m] * s_w[n] * sum_k q_x[m, k] * w[n, k], the
 * activations quantised on the fly with `granularity` (one e4m3 plane: half the tensor
 * work of inferd_fp8_linear), fp32 accumulation in TMEM, bf16 out.  Arguments, layouts and
 * workspace (inferd_fp8_linear_workspace_bytes) as inferd_fp8_linear.
 */
typedef enum { INFERD_FP8_PER_TENSOR = 0, INFERD_FP8_PER_ROW = 1 } inferd_fp8_granularity_t;

INFERD_API int inferd_fp8_quantize_dynamic(const void* x, int32_t x_dtype, void* q, float* scale,
                                           int64_t rows, int64_t k, int32_t granularity,
                                           float* row_amax, void* stream);

INFERD_API int inferd_fp8_dynamic_linear(void* y, const void* x, const void* w_e4m3,
                                         const float* w_scale, int64_t m, int64_t n, int64_t k,
                                         int32_t w_layout, int32_t granularity, void* workspace,
                                         size_t workspace_bytes, void* stream);

/*
 * Decode-step sampling, one row per sequence: temperature + top-p ("nucleus")
 * probabilities and one multinomial draw.  Replaces core/spec_decode.py:14-31
 * nucleus_probs and :34-35 sample_from as called by the scheduler (core/scheduler.py:341-342)
 * and the speculative accept/resample loop (core/spec_decode.py:127-160).
 *
 * inferd_nucleus_sample: logits [rows, logits_stride] (dtype f32/f16/bf16) ->
 *   probs_out [rows, out_stride] fp32 (nullable): softmax(logits / T) with every entry
 *   zeroed whose exclusive cumulative mass in descending order exceeds top_p (equal values
 *   in index order), renormalised; T <= 0 gives a one-hot row at the argmax (the first on
 *   ties);
 *   tokens [rows] int64 (nullable): one draw from that distribution (the argmax when T <= 0).
 * temperatures / top_ps: per-row device arrays, or NULL to use the scalars; top_p > 0.
 * The draw is an inverse CDF in index order over probabilities rounded to multiples of
 * 2^-52, with 64 random bits per row from Philox4x32-10 keyed by seed at counter
 * offset + row; a row with no mass yields -1 and INFERD_ERR_INVALID_ARGUMENT in *error_word.
 * vocab <= 262144.
 */
INFERD_API int inferd_nucleus_sample(float* probs_out, int64_t out_stride, int64_t* tokens,
                                     const void* logits, int32_t dtype, int64_t logits_stride,
                                     int32_t rows, int64_t vocab, const float* temperatures,
                                     float temperature, const float* top_ps, float top_p,
                                     uint64_t seed, uint64_t offset, int32_t* error_word,
                                     void* stream);

/*
 * One multinomial draw per row from non-negative fp32 weights [rows, probs_stride] (need
 * not sum to 1): core/spec_decode.py:34-35 sample_from.  Same draw rule and generator as
 * inferd_nucleus_sample, the weights scaled by a power of two 2^(52 - k) with
 * 2^k >= vocab * max weight before rounding to integers; negative, NaN or infinite weights
 * count as zero and set INFERD_ERR_INVALID_ARGUMENT in *error_word.
 */
INFERD_API int inferd_sample_probs(int64_t* tokens, const float* probs, int64_t probs_stride,
                                   int32_t rows, int64_t vocab, uint64_t seed, uint64_t offset,
                                   int32_t* error_word, void* stream);

/*
 * Speculative decoding's accept / resample step for a batch (core/spec_decode.py:145-161),
 * one launch for every draft position of every sequence.  For sequence b, draft token k
 * (x = proposals[b * proposals_stride + k]) is accepted when u_k <= p_bk[x] / q_bk[x] (fp32
 * division; u_k uniform on the float32 grid of [0, 1) from Philox4x32-10, key seed, counter
 * (offset + b, 1 + k, 0)); at the first rejection one token is drawn from
 * clamp(p_bk - q_bk, 0) -- from p_bk when that has no positive entry -- and the round ends;
 * with all gamma drafts accepted the bonus token is drawn from p_b,gamma.  The draw follows
 * inferd_sample_probs (Philox counter (offset + b, 0, 0)).  p: fp32 [rows][gamma + 1][vocab]
 * at strides (p_seq_stride, p_dist_stride), q: fp32 [rows][gamma][vocab], proposals int64.
 * Outputs: accepted[b] = accepted drafts (0 .. gamma); tokens[b * tokens_stride + 0 ..
 * gamma] = the accepted drafts, the drawn token, then -1.  Replaces one host sync per draft
 * token in the reference's loop.
 */
INFERD_API int inferd_spec_accept(int32_t* accepted, int64_t* tokens, int64_t tokens_stride,
                                  const float* p, int64_t p_seq_stride, int64_t p_dist_stride,
                                  const float* q, int64_t q_seq_stride, int64_t q_dist_stride,
                                  const int64_t* proposals, int64_t proposals_stride,
                                  int32_t rows, int32_t gamma, int64_t vocab, uint64_t seed,
                                  uint64_t offset, int32_t* error_word, void* stream);

/*
 * Output gather over NVLink peer memory (sequence-sharded decode: every rank needs every
 * rank's attention outputs, in rank order).  No counterpart in the reference, which runs
 * on one GPU (core/model_runner.py:32); this replaces an all-gather collective of the
 * per-step outputs.
 *
 * Each rank allocates one peer buffer of 512 + 2 * world * bytes_per_rank bytes with
 * inferd_peer_alloc (zeroed; its CUDA IPC handle, INFERD_IPC_HANDLE_BYTES bytes, goes to
 * every other rank, which maps it with inferd_peer_open).  Layout: uint32 flags[world] at
 * offset 0 (the epoch each source rank last published), uint32 push counters[world] at
 * offset 256 (this rank's own bookkeeping), then slot 0 and slot 1 of world *
 * bytes_per_rank bytes from offset 512.
 *
 * inferd_gather_push copies bytes_per_rank bytes from src (16-byte aligned, a multiple of
 * 16) to dst[d] + rank * bytes_per_rank for every rank d (dst: a device array of world
 * pointers, each rank's current slot), then stores epoch into flags[d][rank] (flags: a
 * device array of world pointers to each rank's flag words) with system-scope release;
 * counters is this rank's own counter array (offset 256 of its buffer).
 * inferd_gather_wait returns, in stream order, once flags[r] >= epoch for every r
 * (wrap-safe), i.e. once every rank's rows for this epoch are in this rank's slot; after
 * timeout_ns (0: 2 s) it records INFERD_ERR_DEVICE_TIMEOUT in *error_word and returns.
 * A rank pushes into a slot again only after its own wait for the following epoch.
 */
#define INFERD_IPC_HANDLE_BYTES 64
INFERD_API int inferd_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
INFERD_API int inferd_peer_open(const void* ipc_handle, void** ptr);
INFERD_API int inferd_peer_close(void* ptr);
INFERD_API int inferd_peer_free(void* ptr);
INFERD_API int inferd_gather_push(const void* src, int64_t bytes_per_rank, void* const* dst,
                                  uint32_t* const* flags, uint32_t* counters, int32_t rank,
                                  int32_t world, uint32_t epoch, void* stream);
INFERD_API int inferd_gather_wait(const uint32_t* flags, int32_t world, uint32_t epoch,
                                  uint64_t timeout_ns, int32_t* error_word, void* stream);

/*
 * The same gather fused into the attention: inferd_paged_attention_gather is
 * inferd_paged_attention (tensor-core path only; other shapes return
 * INFERD_ERR_UNSUPPORTED) whose epilogue also copies every finished (sequence, kv head)
 * block of output rows, as 16-byte vectors, to peer_out[i] + peer_offset + (its index in
 * out) for i < num_peers, each rank's current slot (peer_out: a device array of 16-byte
 * aligned pointers); peer_offset = rank * bytes_per_rank / element size, a multiple of 8
 * elements (INFERD_ERR_INVALID_ARGUMENT otherwise).  inferd_gather_publish then
 * stores epoch into flags[d][rank] for every rank d (system-scope release, after the
 * attention grids on the stream), and inferd_gather_wait orders the consumer as above.
 */
INFERD_API int inferd_paged_attention_gather(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const void* block_tables, int32_t block_table_bytes, int64_t block_table_stride,
    const int32_t* context_lens, int32_t num_seqs, int32_t q_len, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t block_size, int64_t num_blocks,
    int32_t max_context_len, float scale, int32_t dtype, void* workspace, size_t workspace_bytes,
    void* const* peer_out, int32_t num_peers, int64_t peer_offset, int32_t* error_word,
    void* stream);
INFERD_API int inferd_gather_publish(uint32_t* const* flags, int32_t rank, int32_t world,
                                     uint32_t epoch, void* stream);

/*
 * Room beside the attention for a collective on another stream.  The tensor-core
 * attention is a persistent grid that fills every SM and splits the pages statically, so
 * a CTA that cannot start because another kernel holds its SM (an NCCL all-gather of the
 * previous step's outputs) delays the whole call.  After this call, attention grids
 * launched later by this process size themselves for (SM count - sms) SMs, leaving room
 * for a kernel of at most sms CTAs (NCCL's max_ctas).  Process-wide, default 0;
 * 0 <= sms < the SM count of the current device (INFERD_ERR_INVALID_ARGUMENT otherwise).
 * Grids already captured in a CUDA graph keep the size they were captured with.
 * inferd_paged_attention_reserved_sms returns the current value.  No counterpart in the
 * reference, which runs one process on one GPU.
 */
INFERD_API int inferd_paged_attention_reserve_sms(int32_t sms);
INFERD_API int32_t inferd_paged_attention_reserved_sms(void);

#ifdef __cplusplus
}
#endif

#endif /* INFERD_B200_H */
