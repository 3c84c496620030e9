/*
 * needle_b200 -- C ABI of the B200 (sm_100a) attention hot path for needle.
 *
 * Every entry point takes raw device pointers, element strides and sizes,
 * plus the CUDA stream to launch on (a cudaStream_t passed as void*; NULL is
 * the legacy default stream).  Nothing here synchronises the device except
 * nb_device_errors().  Shapes, dtypes and strides are validated on the host
 * and reported as a non-zero status with a message from nb_last_error();
 * nothing is launched in that case.  Kernels never trap: a block id outside
 * the pool or an invalid position is skipped and recorded in a device-side
 * error word that nb_device_errors() returns.
 *
 * Tensor layouts are needle's:
 *   kv_cache     [2, num_blocks, num_kv_heads, block_size, head_dim], dense
 *                (needle/model/runner.py:65-78); index 0 is K, 1 is V.
 *   block_table  [num_seqs, max_blocks_per_seq] int32, row stride given
 *                (needle/model/runner.py:220-235, padded with the last block).
 *   cu_seqlens   [num_seqs + 1] int32 prefix sums of new tokens per sequence.
 *   context_lens [num_seqs] int32, tokens already in the cache
 *                (needle/model/runner.py:204-218).
 * Token-major activations ([T, heads, head_dim]) take a row stride in
 * elements between consecutive tokens; heads are head_dim elements apart.
 */
#ifndef NEEDLE_B200_H
#define NEEDLE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NB_API __attribute__((visibility("default")))
#else
#define NB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define NB_OK 0
#define NB_ERR_INVALID_ARG 1
#define NB_ERR_UNSUPPORTED 2
#define NB_ERR_CUDA 3

/* element types */
#define NB_DTYPE_F32 0
#define NB_DTYPE_F16 1
#define NB_DTYPE_BF16 2

/* bits of the device error word */
#define NB_DEVERR_BLOCK_ID 1u /* a block-table entry outside [0, num_blocks) */
#define NB_DEVERR_POSITION 2u /* a negative context length / position */
#define NB_DEVERR_TIMEOUT 4u  /* a bounded wait on an async copy ran out */

/* ABI version of this header (bumped on any signature change). */
NB_API int nb_abi_version(void);

/* Message of the last non-zero status returned on this thread. */
NB_API const char* nb_last_error(void);

/* Synchronises the current device, returns the device error word in
 * *flags_out and clears it.  Returns NB_ERR_CUDA if the device is in error. */
NB_API int nb_device_errors(unsigned* flags_out);

/*
 * Scatter new K/V tokens into the paged cache.
 * Replaces needle/layers/attention.py:204-246 (_write_kv, prefill) and
 * needle/layers/attention.py:140-154 (the decode KV write).
 * Token i of sequence s goes to position context_lens[s] + i; its block-table
 * column is position / block_size clamped to max_blocks_per_seq - 1 (:235);
 * when the clamp makes several tokens of one sequence share a slot the last
 * one wins.  cu_seqlens == NULL means one token per sequence (decode):
 * num_tokens must then equal num_seqs.  Byte-exact copy.
 */
NB_API int nb_store_kvcache(const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                     void* kv_cache, int num_blocks, int num_kv_heads, int block_size,
                     int head_dim, const int32_t* block_table, int64_t block_table_stride,
                     int max_blocks_per_seq, const int32_t* cu_seqlens,
                     const int32_t* context_lens, int num_seqs, int num_tokens, int dtype,
                     void* stream);

/*
 * Slot table of one forward: slots[t] = block * block_size + offset of new
 * token t in the paged cache, or -1 when the token is not written (a block id
 * outside [0, num_blocks) or a negative context length, both recorded in the
 * device error word; or an earlier token on a clamped slot that a later token
 * of the same sequence overwrites).  Same index math, clamp and
 * last-token-wins rule as nb_store_kvcache, which restates
 * needle/layers/attention.py:214-240 (prefill) and :140-154 (decode).
 * needle recomputes these positions in every layer; here the table is built
 * once per forward and read by every layer's nb_store_kvcache_slots /
 * nb_rope_store_kvcache_slots.  cu_seqlens == NULL: one token per sequence.
 */
NB_API int nb_slot_mapping(const int32_t* block_table, int64_t block_table_stride,
                           int max_blocks_per_seq, const int32_t* cu_seqlens,
                           const int32_t* context_lens, int num_seqs, int num_tokens,
                           int block_size, int num_blocks, int32_t* slots, void* stream);

/*
 * nb_store_kvcache with the positions taken from a slot table
 * (nb_slot_mapping): token t's K/V rows go to block slots[t] / block_size,
 * row slots[t] % block_size; slots[t] < 0 is skipped.  Replaces
 * needle/layers/attention.py:140-154 and :204-246 like nb_store_kvcache.
 * Rows must be 16-byte aligned.  Byte-exact copy.
 */
NB_API int nb_store_kvcache_slots(const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                                  void* kv_cache, int num_blocks, int num_kv_heads,
                                  int block_size, int head_dim, const int32_t* slots,
                                  int num_tokens, int dtype, void* stream);

/*
 * nb_rope_store_kvcache with the positions taken from a slot table: q is
 * rotated in place, k rotated and written to the cache (and back into k when
 * write_k_back != 0), v copied to the cache.  Replaces
 * needle/layers/attention.py:88 (_apply_rope) + :140-154 or :204-246.  Same
 * rounding as nb_rope (bit-identical to the reference).  Rows must be
 * 16-byte aligned.
 */
NB_API int nb_rope_store_kvcache_slots(void* q, int64_t q_stride, int num_q_heads, void* k,
                                       int64_t k_stride, const void* v, int64_t v_stride,
                                       const void* cos, const void* sin, int64_t cs_stride,
                                       void* kv_cache, int num_blocks, int num_kv_heads,
                                       int block_size, int head_dim, const int32_t* slots,
                                       int num_tokens, int write_k_back, int dtype,
                                       void* stream);

/*
 * In-place NeoX rotary embedding of q [T, num_q_heads, D] and k
 * [T, num_kv_heads, D] with per-token tables cos/sin [T, D] (row stride
 * cs_stride).  Replaces needle/layers/attention.py:277-288 (_apply_rope):
 * x*cos + rotate_half(x)*sin with the result of each multiply and of the add
 * rounded to the storage dtype, so the output is bit-identical to the
 * reference.  k may be NULL (num_kv_heads ignored).
 */
NB_API int nb_rope(void* q, int64_t q_stride, int num_q_heads, void* k, int64_t k_stride,
            int num_kv_heads, const void* cos, const void* sin, int64_t cs_stride, int num_tokens,
            int head_dim, int dtype, void* stream);

/*
 * nb_rope followed by nb_store_kvcache in one launch: q is rotated in place,
 * k is rotated and written to the cache (and back into k when
 * write_k_back != 0), v is copied to the cache.  Replaces the sequence
 * needle/layers/attention.py:88 (_apply_rope) + :140-154 or :204-246.
 */
NB_API int nb_rope_store_kvcache(void* q, int64_t q_stride, int num_q_heads, void* k, int64_t k_stride,
                          const void* v, int64_t v_stride, const void* cos, const void* sin,
                          int64_t cs_stride, void* kv_cache, int num_blocks, int num_kv_heads,
                          int block_size, int head_dim, const int32_t* block_table,
                          int64_t block_table_stride, int max_blocks_per_seq,
                          const int32_t* cu_seqlens, const int32_t* context_lens, int num_seqs,
                          int num_tokens, int write_k_back, int dtype, void* stream);

/*
 * Split-K plan for nb_paged_decode: pages (KV blocks) per split and the
 * number of splits per sequence that the workspace must hold, chosen from
 * the batch shape and the block-table width only (no device reads).
 */
NB_API int nb_paged_decode_plan(int num_seqs, int num_kv_heads, int max_blocks_per_seq, int block_size,
                         int* pages_per_split, int* max_splits);

/* Bytes of workspace nb_paged_decode needs for this shape and split count. */
NB_API size_t nb_paged_decode_workspace_size(int num_seqs, int num_q_heads, int head_dim,
                                      int max_splits);

/*
 * Paged decode attention: for every sequence s and query head j, attention
 * of q[s, j] over the first context_lens[s] + 1 cached tokens of KV head
 * j / (num_q_heads / num_kv_heads), scaled by `scale`.
 * Replaces needle/layers/attention.py:291-310 (_decode_pytorch) and
 * :161-197 (_decode_flashinfer).  Split-K: each split of pages_per_split
 * pages is one CTA per (split, kv head, sequence) writing fp32 partials to
 * `workspace`; a separate merge kernel combines the splits.  Any group size
 * num_q_heads / num_kv_heads (power of two or not) is supported.
 * The caller allocates the workspace (nb_paged_decode_workspace_size).
 */
NB_API int nb_paged_decode(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                    const void* kv_cache, int num_blocks, int num_kv_heads, int block_size,
                    int head_dim, int num_q_heads, const int32_t* block_table,
                    int64_t block_table_stride, int max_blocks_per_seq,
                    const int32_t* context_lens, int num_seqs, float scale, void* out,
                    int64_t out_stride_seq, int64_t out_stride_head, void* workspace,
                    size_t workspace_bytes, int pages_per_split, int dtype, void* stream);

/*
 * Size in bytes of the fixed split-K scratch that nb_paged_decode_noalloc
 * uses (16 MiB, held in the library's own device memory on every GPU that
 * loads the library, for the life of the process).
 */
#define NB_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/*
 * nb_paged_decode for callers that cannot allocate device memory: no
 * workspace argument.  This entry point has no counterpart in needle (needle
 * allocates its decode workspace with torch, attention.py:178-184); it exists
 * for callers without a device allocator of their own (an FFI host with no
 * torch), callers that must not call cudaMalloc between launches (it can
 * synchronise the device), and callers whose device memory is fixed at
 * start-up.  The split-K partials live in one fixed array of
 * NB_NOALLOC_SCRATCH_BYTES inside the library; a shape whose partials do not
 * fit is rejected with NB_ERR_INVALID_ARG and a message.  The first call on
 * each device looks up the array's device address (make it before any
 * stream capture).  All calls share the array: calls that overlap on the GPU
 * race and must be serialised by the caller.  Allocates nothing.
 */
NB_API int nb_paged_decode_noalloc(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                                   const void* kv_cache, int num_blocks, int num_kv_heads,
                                   int block_size, int head_dim, int num_q_heads,
                                   const int32_t* block_table, int64_t block_table_stride,
                                   int max_blocks_per_seq, const int32_t* context_lens,
                                   int num_seqs, float scale, void* out, int64_t out_stride_seq,
                                   int64_t out_stride_head, int pages_per_split, int dtype,
                                   void* stream);

/*
 * Causal prefill attention over each sequence's new tokens, q [T, Hq, D],
 * k/v [T, Hkv, D] (post-RoPE, token-major, row strides given), output
 * [T, Hq, D].  Replaces needle/layers/attention.py:120-134 (_prefill_pytorch)
 * and :109-118 (_prefill_flashinfer): within sequence s token i attends to
 * tokens 0..i of the same sequence, query head j to KV head j / group.
 * bf16 / fp16 with head_dim 64 or 128, 16-byte aligned q, k, v and out and
 * row strides of a multiple of 16 bytes run on the tcgen05 kernel; anything
 * else (fp32, other head dims, unaligned rows) runs a slower SIMT kernel with
 * the same semantics.
 */
NB_API int nb_prefill_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                         const void* v, int64_t v_stride, int num_q_heads, int num_kv_heads,
                         int head_dim, const int32_t* cu_seqlens, int num_seqs, int num_tokens,
                         int max_seqlen, float scale, void* out, int64_t out_stride, int dtype,
                         void* stream);

/*
 * RMSNorm of x [T, hidden]: y = weight * (x * rsqrt(mean(x^2) + eps)), with
 * the mean of squares in fp32 and the rounding points of
 * needle/layers/norm.py:14-17.
 */
NB_API int nb_rmsnorm(const void* x, int64_t x_stride, const void* weight, void* out,
               int64_t out_stride, int num_tokens, int hidden, float eps, int dtype,
               void* stream);

/*
 * Residual add fused with RMSNorm: h = residual + x (rounded to dtype),
 * residual_out = h, out = RMSNorm(h).  Replaces the decoder-layer sequence
 * needle/model/llama.py:67-70 (and :72 + the next layer's :62).
 * residual_out may alias residual; out may alias x.
 */
NB_API int nb_fused_add_rmsnorm(const void* x, int64_t x_stride, const void* residual,
                         int64_t residual_stride, const void* weight, void* out,
                         int64_t out_stride, void* residual_out, int64_t residual_out_stride,
                         int num_tokens, int hidden, float eps, int dtype, void* stream);

/*
 * Copy whole KV blocks between two paged caches of num_layers layers, e.g.
 * the device cache and a pinned host cache (swap-out / swap-in), in one
 * launch.  Replaces needle/model/runner.py:175-192 (_swap_kv_blocks, one
 * .to() per block per layer).  src_caches / dst_caches: host arrays of
 * num_layers cache base pointers (device memory or pinned host memory, both
 * addressable by the GPU); block_pairs: num_pairs (src block, dst block)
 * int32 pairs in GPU-addressable memory; block_bytes: bytes of one block's
 * K (or V) half = num_kv_heads * block_size * head_dim * element size.
 * Out-of-range block ids are skipped and recorded (NB_DEVERR_BLOCK_ID).
 */
NB_API int nb_swap_kv_blocks(const void* const* src_caches, void* const* dst_caches,
                             int num_layers, const int32_t* block_pairs, int num_pairs,
                             int64_t src_num_blocks, int64_t dst_num_blocks, int64_t block_bytes,
                             void* stream);

/*
 * CUDA IPC plumbing for the fused TP all-reduce: export the allocation that
 * contains dev_ptr (64-byte handle + offset of dev_ptr inside it), map a
 * peer's handle (the caller adds the offset), unmap.
 */
NB_API int nb_ipc_handle(const void* dev_ptr, void* handle_out, uint64_t* offset_out);
NB_API int nb_ipc_open(const void* handle, void** dev_ptr_out);
NB_API int nb_ipc_close(void* dev_ptr);

/*
 * Tensor-parallel all-reduce of the row-parallel projection output fused
 * with the decoder's residual add and RMSNorm, over NVLink peer memory.
 * Replaces needle/layers/linear.py:92-98 (dist.all_reduce of o_proj /
 * down_proj) + needle/model/llama.py:67-72 (residual add, RMSNorm).
 * partial: this rank's partial sums [T, hidden]; residual: the residual
 * [T, hidden], updated in place; out: the normalised rows [T, hidden] (all
 * three local).  recv / gather: world-long arrays of peer-mapped pointers
 * (index = rank) to each rank's receive slots [2][world][slot_rows][hidden]
 * and gather slots [2][world][slot_rows][2][hidden], filled with 0xFF bytes
 * before first use.  epochs: this rank's zero-initialised
 * NB_TP_EPOCH_WORDS uint32 (device): per-row call counters, then the
 * communicator's status word at index NB_TP_STATUS_WORD.  host_status:
 * NULL, or a word of pinned host memory that the kernel sets to 1 when a wait
 * on a peer times out (the host reads it without a device sync).  After a
 * timeout the status word is set and every later call returns without
 * touching the buffers, until the caller refills recv/gather with 0xFF and
 * zeroes epochs (status word included) on every rank.  Every owner sums the
 * partials in rank order, so all ranks hold identical bits.
 * ceil(T / world) <= min(1024, slot_rows), hidden % 8 == 0 and <= 8192,
 * bf16/fp16, 16-byte aligned buffers.  All ranks must make the same sequence
 * of calls.
 */
#define NB_TP_EPOCH_WORDS 2080
#define NB_TP_STATUS_WORD 2048
NB_API int nb_tp_allreduce_add_rmsnorm(const void* partial, void* const* recv,
                                       void* const* gather, int slot_rows, void* out,
                                       void* residual, unsigned* epochs, unsigned* host_status,
                                       int rank, int world, const void* weight, int num_tokens,
                                       int hidden, float eps, int dtype, void* stream);

/*
 * Upper bound in nanoseconds of each wait that nb_tp_allreduce_add_rmsnorm
 * makes on a peer (0 = the default of 2 s; at most 60 s).  Read at every
 * launch, so a captured CUDA graph keeps the value of its capture.  Part of
 * the failure handling that replaces NCCL's timeout on needle's all-reduce
 * (needle/layers/linear.py:92-98 relies on the process group's timeout).
 */
NB_API int nb_tp_set_wait_limit_ns(uint64_t ns);

/*
 * SwiGLU activation over a fused gate/up projection: gate_up is [T, 2*I]
 * (gate in columns [0, I), up in [I, 2I)), out[T, I] = silu(gate) * up with
 * the rounding points of needle/model/llama.py:37 (F.silu, then the
 * multiply, each rounded to the storage dtype).
 */
NB_API int nb_silu_mul(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                       int num_tokens, int intermediate, int dtype, void* stream);

/*
 * Sampling for a whole decode step in one launch, one row of logits
 * [num_rows, vocab] (row stride given) per CTA.  Replaces
 * needle/model/sampler.py:24-46 (a per-row loop with one host read per row).
 * temperature, top_k, top_p and uniforms are per-row device arrays:
 *   temperature == 0: greedy, the first index of the maximal logit (NaN
 *     counts as maximal, as torch.argmax);
 *   otherwise x = logit / temperature (rounded to the logits' dtype); top_k >
 *     0 keeps x >= the top_k-th largest x; top_p < 1 then keeps, in
 *     descending order of x (ties in index order), each token whose
 *     probability mass before it (softmax over the kept tokens, each
 *     probability rounded to the logits' dtype, summed in fp32) is at most
 *     top_p; one token is drawn by inverse CDF in vocabulary order at
 *     uniforms[row] in [0, 1).
 * token_ids: [num_rows] int64 (device).  filtered: NULL, or [num_rows, vocab]
 * of the logits' dtype receiving each sampled row's filtered logits (removed
 * tokens -inf; greedy rows untouched).
 */
NB_API int nb_sample(const void* logits, int64_t row_stride, int num_rows, int vocab,
                     const float* temperature, const int32_t* top_k, const float* top_p,
                     const float* uniforms, void* filtered, int64_t filtered_stride,
                     int64_t* token_ids, int dtype, void* stream);

/*
 * Paged prefill: causal attention of the new tokens of each sequence over
 * the sequence's whole context — the context_lens[s] tokens already cached
 * and the new tokens themselves — read from the paged cache
 * [2, num_blocks, num_kv_heads, 16, head_dim] through the block table (the
 * new tokens' K/V must have been written first, e.g. by
 * nb_rope_store_kvcache_slots).  Query row i of sequence s sits at position
 * context_lens[s] + i and sees keys 0 .. context_lens[s] + i.  With every
 * context_lens[s] == 0 the result is nb_prefill_attention's.  This is the
 * continuation case needle's own prefill does not handle (it attends over
 * the new tokens only: needle/layers/attention.py:101-134, and its TODO.md
 * lists the gap); decode attends over the cached tokens the same way
 * (attention.py:291-310), so a chunk of n new tokens equals n decode steps;
 * as in decode, a context longer than max_blocks * 16 keys sees only the
 * table's pages.  bf16 / fp16, head_dim 64 or 128, tcgen05;
 * NB_ERR_UNSUPPORTED otherwise.
 */
NB_API int nb_prefill_attention_paged(const void* q, int64_t q_stride, const void* kv_cache,
                                      int num_blocks, int num_kv_heads, const int32_t* block_table,
                                      int64_t bt_stride, int max_blocks,
                                      const int32_t* context_lens, int num_q_heads, int head_dim,
                                      const int32_t* cu_seqlens, int num_seqs, int num_tokens,
                                      int max_seqlen, float scale, void* out, int64_t out_stride,
                                      int dtype, void* stream);

/*
 * Dense projection of a decode step: y[M, N] = x[M, K] . weight[N, K]^T
 * (+ bias[N] when bias is not NULL), fp32 accumulation, output rounded to
 * the input dtype (bf16 or fp16).  Replaces the F.linear of needle's
 * ColumnParallelLinear / RowParallelLinear (needle/layers/linear.py:44,
 * :92) for batches of at most 256 rows; x and weight rows 16-byte aligned
 * (K, x_stride and w_stride multiples of 8).  Returns NB_ERR_UNSUPPORTED
 * for shapes outside that (the caller keeps its library GEMM).
 */
NB_API int nb_linear(const void* x, int64_t x_stride, const void* weight, int64_t w_stride,
                     const void* bias, void* y, int64_t y_stride, int M, int N, int K, int dtype,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NEEDLE_B200_H */
