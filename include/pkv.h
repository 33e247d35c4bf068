/*
 * pkv.h -- C ABI of the B200 (sm_100a) paged-KV hot path for mini-inference.
 *
 * Every entry point takes plain pointers, sizes and strides (in elements),
 * returns an int status (PKV_OK == 0) and never allocates device memory:
 * the caller owns the KV pool, the inputs, the outputs and any workspace.
 * Kernels are enqueued on the given stream and never synchronise the host.
 *
 * The reference (Ham12-3/mini-inference) is pure Python/PyTorch; each entry
 * point names the reference code it replaces. A Python binding (ctypes) is
 * in mini_inference_b200/_lib.py.
 */
#ifndef PKV_H_
#define PKV_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PKV_API __attribute__((visibility("default")))
#else
#define PKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* pkv_stream_t; /* same type as cudaStream_t; NULL = legacy default stream */

/* ------------------------------------------------------------------ status */
enum pkv_status {
  PKV_OK = 0,
  PKV_ERR_INVALID_ARGUMENT = 1,   /* null pointer, bad size, stride, alignment or dtype */
  PKV_ERR_OUT_OF_RANGE = 2,       /* block id, slot or position outside the pool / table */
  PKV_ERR_WORKSPACE = 3,          /* workspace smaller than pkv_decode_workspace_bytes() */
  PKV_ERR_CUDA = 4,               /* a CUDA runtime call failed (see pkv_last_cuda_error) */
  PKV_ERR_NO_BLOCKS = 5,          /* "not enough free KV cache blocks" (engine/kv_cache.py:520) */
  PKV_ERR_DOUBLE_FREE = 6,        /* "slot freed twice" (engine/kv_cache.py:556) */
  PKV_ERR_UNKNOWN_SLOT = 7,       /* slot id that does not own a block table */
  PKV_ERR_UNSUPPORTED = 8,        /* head_dim / group size / dtype combination not built */
  PKV_ERR_TIMEOUT = 9,            /* a bounded device-side wait gave up */
  PKV_ERR_EMPTY_PROMPT = 10,      /* "prompt is empty" (engine/scheduler.py:57-58) */
  PKV_ERR_PROMPT_TOO_LONG = 11    /* prompt_len >= max_model_len (engine/scheduler.py:59-63) */
};

/* Human-readable name of a status code (static string). */
PKV_API const char* pkv_status_string(int status);
/* Text of the last CUDA error seen by this library on the calling thread. */
PKV_API const char* pkv_last_cuda_error(void);
/* Library version, e.g. 0x000100 for 0.1.0. */
PKV_API int pkv_version(void);

/* ------------------------------------------------------------------ KV pool */
enum pkv_dtype { PKV_F16 = 0, PKV_BF16 = 1 };

/*
 * One KV pool, the reference's layout (engine/kv_cache.py:411-443):
 *   k, v: [num_layers, num_blocks_total, num_kv_heads, block_size, head_dim], contiguous,
 * where num_blocks_total includes the scratch block that CUDA-graph padding
 * rows write to (engine/kv_cache.py:426-429).
 */
typedef struct pkv_pool {
  void* k;
  void* v;
  int32_t num_layers;
  int32_t num_blocks_total;
  int32_t num_kv_heads;
  int32_t block_size;
  int32_t head_dim;
  int32_t dtype; /* enum pkv_dtype */
} pkv_pool;

/*
 * Block tables as the kernels read them: int32 block ids, row r at
 * block_tables + r * stride, `cols` entries per row. With seq_rows == NULL,
 * batch entry b reads row b (a padded [batch, cols] table, as the reference
 * builds at engine/kv_cache.py:606-607). With seq_rows, batch entry b reads row
 * seq_rows[b] of a device-resident mirror indexed by slot; seq_rows[b] < 0 marks
 * a CUDA-graph padding row, which reads and writes only the scratch block.
 */
typedef struct pkv_tables {
  const int32_t* block_tables;
  int64_t stride;
  int32_t rows;
  int32_t cols;
  const int32_t* seq_rows;
} pkv_tables;

/*
 * KV append: scatter n_tokens new K/V rows into the pool through slot_mapping
 * (slot = block * block_size + offset; a negative slot skips the row).
 * Row t, head h of k_new starts at k_new + t * tok_stride + h * head_stride
 * (head_dim elements contiguous); v_new uses the same strides.
 * Replaces the index_put scatters `k_layer[write_blocks, :, write_offsets] = k`
 * of engine/kv_cache.py:613-614 (decode) and :288-289 (packed prefill), and
 * engine/cuda_graphs.py:82-83.
 * status_dev (optional) receives PKV_ERR_OUT_OF_RANGE if a slot is past the pool.
 */
PKV_API int pkv_kv_append(const pkv_pool* pool, int32_t layer, const void* k_new, const void* v_new,
                  int64_t n_tokens, int64_t tok_stride, int64_t head_stride, const int64_t* slot_mapping,
                  int32_t* status_dev, pkv_stream_t stream);

/*
 * Paged decode attention, one new token per sequence, optionally fused with
 * its KV append. Replaces PagedDecodeContext.attend (engine/kv_cache.py:611-620)
 * = append + block gather + decode_attention (engine/model.py:126-147), and
 * _GraphDecodeContext.attend (engine/cuda_graphs.py:79-92).
 *
 *   q       : row b, query head h at q + b*q_stride_b + h*q_stride_h (head_dim contiguous)
 *   out     : row b, query head h at out + b*out_stride_b + h*out_stride_h
 *   k_new/v_new (both NULL = no append): row b, kv head j at k_new + b*kv_stride_b + j*kv_stride_h;
 *             written to slot_mapping[b] and attended at position context_lens[b]-1
 *   tables  : see pkv_tables
 *   context_lens[b]: keys row b attends to (its position + 1), 1..tables->cols*block_size
 *   scale   : softmax scale (the reference uses 1/sqrt(head_dim))
 *   flags   : PKV_DECODE_INPUTS_READY or 0 (see below)
 *   workspace: >= pkv_decode_workspace_bytes(...) bytes, 256-byte aligned, zeroed once
 *             before first use; every call leaves it ready for the next, whatever the
 *             next call's batch or table width. Calls that share a workspace must not
 *             overlap on the GPU.
 * Supported: fp16 / bf16, block_size 16, head_dim 64 or 128, num_kv_heads 1, 2, 4 or 8,
 * query heads per KV head <= 16, batch <= 1024; anything else returns PKV_ERR_UNSUPPORTED.
 * Query head h reads KV head h / (num_q_heads / num_kv_heads), as the reference's regrouping.
 */
PKV_API int pkv_decode_attention(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t batch,
                         int32_t num_q_heads, void* out, int64_t out_stride_b, int64_t out_stride_h,
                         const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* k_new,
                         const void* v_new, int64_t kv_stride_b, int64_t kv_stride_h,
                         const int64_t* slot_mapping, const int32_t* context_lens, float scale,
                         int32_t flags, void* workspace, int64_t workspace_bytes, int32_t* status_dev,
                         pkv_stream_t stream);

/*
 * pkv_decode_attention with the rotary position embedding fused in: q, the new k and the new
 * v come straight from the qkv_proj output, and q and k are rotated inside the kernel at
 * position context_lens[b] - 1, bit-identical to the reference's apply_rope on the same
 * tables (r(r(x * cos) + r(rotate_half(x) * sin)) per element). Replaces, for a decode step,
 * pkv_rope_append (rotation) followed by pkv_decode_attention (append + attention): one
 * launch per layer instead of two (engine/model.py:241-250 + engine/kv_cache.py:611-620).
 *   qkv   : row b [q (Hq*d) | k (Hkv*d) | v (Hkv*d)] at qkv + b*qkv_stride (elements)
 *   cos_table, sin_table : [max_positions, d] in the storage dtype (as pkv_rope_append)
 *   slot_mapping : required (the rotated k and v are appended there)
 * Everything else is pkv_decode_attention's; a position past the tables is reported in status.
 */
PKV_API int pkv_decode_attention_rope(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t batch,
                              int32_t num_q_heads, void* out, int64_t out_stride_b, int64_t out_stride_h,
                              const void* qkv, int64_t qkv_stride, const void* cos_table, const void* sin_table,
                              int64_t max_positions, const int64_t* slot_mapping, const int32_t* context_lens,
                              float scale, int32_t flags, void* workspace, int64_t workspace_bytes,
                              int32_t* status_dev, pkv_stream_t stream);

/* pkv_decode_attention flags */
enum {
  /* context_lens, the block tables / seq_rows and every cached K/V row the call reads were
   * complete before the previous kernel in the stream began (only q, k_new and v_new may come
   * from it). The kernel then resolves blocks and starts its first K/V copies before waiting
   * for that kernel (programmatic dependent launch). E.g. layers after the first of a decode
   * step whose metadata was built at the start of the step. */
  PKV_DECODE_INPUTS_READY = 1
};

/* Workspace bytes pkv_decode_attention needs for these sizes. */
PKV_API int64_t pkv_decode_workspace_bytes(int32_t batch, int32_t num_kv_heads, int32_t max_blocks_per_seq,
                                   int32_t block_size, int32_t head_dim, int32_t num_q_heads);

/*
 * Zero a decode workspace's ticket counters on `stream` (its first 4 KB). Every call leaves
 * them at zero; after a call that reported an error (a timed-out wait, a refused unit) the
 * caller resets them before reusing the workspace, so a stale ticket cannot make a later
 * call merge the wrong chunks. No counterpart in the reference (it keeps no device state
 * between steps).
 */
PKV_API int pkv_decode_reset_workspace(void* workspace, int64_t workspace_bytes, pkv_stream_t stream);

/* Size of the device array that pkv_decode_attention_static uses as its workspace. On a
 * 148-SM B200 it holds every supported shape except 8 KV heads with more than 8 query heads
 * each at head_dim 128 (which needs 20 MB): see pkv_decode_attention_static. */
#define PKV_DECODE_STATIC_SCRATCH_BYTES (16 * 1024 * 1024)

/*
 * pkv_decode_attention without a workspace argument; it allocates nothing. No counterpart
 * in the reference, which gathers each step into fresh tensors: this is for callers that
 * reach the library over a plain C FFI from a process whose device memory another
 * allocator owns, and so cannot get a workspace buffer mid-step.
 * Arguments, results and status words are those of pkv_decode_attention. Its workspace is
 * one file-scope device array of PKV_DECODE_STATIC_SCRATCH_BYTES per device:
 *   - what a launch needs depends on the model's shape (KV heads, query heads per KV head,
 *     head_dim) and the GPU's SM count, not on the batch: 4 KB of tickets plus
 *     2 * CTAs * kv_heads * (8 or 16 rows) * (head_dim + 4) floats. A shape that needs more
 *     (on a 148-SM B200: 8 KV heads, group > 8, head_dim 128) returns PKV_ERR_WORKSPACE for
 *     every call and launches nothing;
 *   - every call on a device shares it, so calls that overlap on the GPU (other streams,
 *     other host threads) race and must be serialised by the caller;
 *   - the first call on a device looks the array up and clears it on `stream` (the current
 *     device must be the stream's); make that call before any stream capture.
 */
PKV_API int pkv_decode_attention_static(const pkv_pool* pool, int32_t layer, const pkv_tables* tables,
                                int32_t batch, int32_t num_q_heads, void* out, int64_t out_stride_b,
                                int64_t out_stride_h, const void* q, int64_t q_stride_b, int64_t q_stride_h,
                                const void* k_new, const void* v_new, int64_t kv_stride_b,
                                int64_t kv_stride_h, const int64_t* slot_mapping, const int32_t* context_lens,
                                float scale, int32_t flags, int32_t* status_dev, pkv_stream_t stream);

/* Zero the current device's static decode scratch tickets on `stream` (set-up included, as
 * on a first call): what pkv_decode_reset_workspace does for a caller workspace, for use
 * after a pkv_decode_attention_static call that reported an error. */
PKV_API int pkv_decode_static_reset(pkv_stream_t stream);
/* Device address and size of the current device's static decode scratch (set-up included),
 * for callers that inspect or clear it themselves; it is the array's real device address,
 * found with cudaGetSymbolAddress. */
PKV_API int pkv_decode_static_scratch(void** address, int64_t* bytes, pkv_stream_t stream);

/*
 * Packed (varlen) prefill attention over the paged cache, prefix-cache hits included.
 * Replaces PackedPrefillContext.attend (engine/kv_cache.py:283-297) after its append:
 * sequence s owns packed tokens cu_seqlens[s]..cu_seqlens[s+1]-1, which sit at
 * positions starts[s] + i; each attends to its own sequence's keys 0..position,
 * read from the pool (the new tokens must already be appended, pkv_kv_append).
 *   q   : token t, query head h at q + t*q_stride_t + h*q_stride_h
 *   out : token t, query head h at out + t*out_stride_t + h*out_stride_h
 *   tables : see pkv_tables (one row per sequence)
 */
PKV_API int pkv_prefill_attention(const pkv_pool* pool, int32_t layer, const pkv_tables* tables, int32_t num_seqs,
                          const int32_t* cu_seqlens, const int32_t* starts, int32_t max_new_tokens,
                          int32_t num_q_heads, void* out, int64_t out_stride_t, int64_t out_stride_h,
                          const void* q, int64_t q_stride_t, int64_t q_stride_h, float scale,
                          int32_t* status_dev, pkv_stream_t stream);

/*
 * Rotary position embedding of q and k, fused with the KV append (the "qkv-post"
 * step). Replaces the split and head views of Attention.forward, the table lookup of
 * RotaryEmbedding.forward and apply_rope (engine/model.py:201-224, 236-249) and, with
 * slot_mapping, the index_put append of the new K/V rows (engine/kv_cache.py:288-289,
 * 613-614). q and k come out bit-identical to the reference's eager ops on the same
 * tables: r(r(x*cos) + r(rotate_half(x)*sin)), each step in float32, rounded once.
 *
 *   qkv   : token t's row [q (Hq*d) | k (Hkv*d) | v (Hkv*d)] at qkv + t*qkv_stride
 *           (the qkv_proj output, bias included), storage dtype of the pool
 *   positions : int64 [n_tokens], each in [0, max_positions)
 *   cos_table, sin_table : [max_positions, d] in the storage dtype (the reference's
 *           float32 tables cast to it, engine/model.py:190-210)
 *   q_out : token t, query head h at q_out + t*q_out_stride_t + h*q_out_stride_h
 *   k_out (NULL = not written): token t, kv head j at k_out + t*k_out_stride_t + j*k_out_stride_h
 *   slot_mapping (NULL = no append): rotated k and v of token t written to the pool at
 *           (layer, slot); a negative slot is skipped. At least one of k_out and
 *           slot_mapping must be given. The decode path passes k_out and lets
 *           pkv_decode_attention append (k_new = k_out, v_new = the v columns of qkv).
 * Out-of-range positions or slots are reported in status (PKV_ERR_OUT_OF_RANGE).
 */
PKV_API int pkv_rope_append(const pkv_pool* pool, int32_t layer, const void* qkv, int64_t qkv_stride,
                    int64_t n_tokens, int32_t num_q_heads, const int64_t* positions, const void* cos_table,
                    const void* sin_table, int64_t max_positions, void* q_out, int64_t q_out_stride_t,
                    int64_t q_out_stride_h, void* k_out, int64_t k_out_stride_t, int64_t k_out_stride_h,
                    const int64_t* slot_mapping, int32_t* status_dev, pkv_stream_t stream);

/* ------------------------------------------------------------------ greedy LM head */
/*
 * The LM head fused with greedy selection: for each of the batch's hidden rows,
 *   token_ids[b] = argmax_v round(hidden[b] . weight[v])
 * with the logit rounded to the model dtype (fp32 accumulation) and the smallest index
 * among equal maxima (NaN counts as the largest), which is what the reference computes for
 * an all-greedy batch: Qwen2ForCausalLM.compute_logits = F.linear(hidden, weight) in the
 * model dtype, .float(), then Sampler's logits.argmax(dim=-1) (engine/model.py:321-323,
 * engine/engine.py:97-123, engine/sampler.py:27-31) -- without writing the [B, vocab]
 * logits. max_logits (NULL = not written) receives each row's largest rounded logit.
 *
 *   hidden : [batch, hidden_size] at hidden + b*hidden_stride (elements), 16-byte aligned
 *   weight : [vocab, hidden_size] at weight + v*weight_stride (the tied embedding or lm_head)
 *   dtype  : PKV_F16 or PKV_BF16 (both operands)
 *   batch <= 256, hidden_size a multiple of 64, strides multiples of 8 elements
 *   workspace : pkv_lm_head_argmax_workspace_bytes(batch) bytes, zeroed once before the
 *           first call; every call leaves it zeroed (one workspace per stream)
 *   flags  : PKV_LM_WEIGHT_READY or 0: the weight was not written by the kernel launched
 *           just before on this stream, so its first stages may be read while that kernel
 *           drains (programmatic dependent launch)
 * Unsupported shapes return PKV_ERR_UNSUPPORTED; a timed-out device wait sets status.
 */
enum { PKV_LM_WEIGHT_READY = 1 };
PKV_API int64_t pkv_lm_head_argmax_workspace_bytes(int32_t batch);
PKV_API int pkv_lm_head_argmax(const void* hidden, int64_t hidden_stride, int32_t batch, const void* weight,
                       int64_t weight_stride, int32_t vocab, int32_t hidden_size, int32_t dtype,
                       int64_t* token_ids, float* max_logits, void* workspace, int64_t workspace_bytes,
                       int32_t flags, int32_t* status_dev, pkv_stream_t stream);

/* ------------------------------------------------------------------ decoder-layer glue */
/*
 * The elementwise steps of the Qwen2 decoder layer around the attention call, one launch
 * each instead of the reference's eager chains (engine/model.py:162-166 RMSNorm,
 * :262-264 the MLP's silu(gate) * up, :278-280 the residual adds).
 *
 * pkv_add_rms_norm, per row of [rows, hidden] (strides in elements):
 *   h   = residual_in ? round(x + residual_in) : x      (the residual add, x = the block output)
 *   residual_out (NULL = not written) receives h; it may be residual_in itself (in place)
 *   out = round(weight * round(h * rsqrt(mean(h^2) + eps)))   (statistics in float32)
 * The add and every rounding are the reference's; the float32 sum of squares runs in its
 * own order. out may alias x. hidden <= 8192 (any multiple of 8 up to 65536 when every
 * row start is 16-byte aligned).
 *
 * pkv_silu_mul, per row of gate_up = [rows, 2 * intermediate] (gate | up):
 *   out[:, j] = round(round(silu(gate[:, j])) * up[:, j]),  silu(g) = g / (1 + exp(-g)) in float32
 *
 * dtype: PKV_F16 or PKV_BF16 for every operand. 16-byte accesses when the rows allow
 * them, 2-byte ones otherwise.
 */
PKV_API int pkv_add_rms_norm(int32_t dtype, const void* x, int64_t x_stride, const void* residual_in,
                             int64_t residual_in_stride, void* residual_out, int64_t residual_out_stride,
                             const void* weight, void* out, int64_t out_stride, int64_t rows, int32_t hidden,
                             float eps, pkv_stream_t stream);
/*
 * pkv_add_rms_norm with x given as split-K partial sums of the block's output projection:
 * partials[s][r][c] at partials + s*split_stride + r*row_stride + c (float32, splits >= 1),
 * as a GEMM cut along K leaves them (e.g. a batched GEMM with float32 output). x = round(sum
 * of the splits in order), the projection's output as F.linear would round it; the rest is
 * pkv_add_rms_norm's. Lets a long-K projection of a decode batch (down_proj, K = 4864) run on
 * more SMs without a separate reduction launch.
 */
PKV_API int pkv_add_rms_norm_partials(int32_t dtype, const float* partials, int64_t row_stride, int32_t splits,
                                      int64_t split_stride, const void* residual_in, int64_t residual_in_stride,
                                      void* residual_out, int64_t residual_out_stride, const void* weight,
                                      void* out, int64_t out_stride, int64_t rows, int32_t hidden, float eps,
                                      pkv_stream_t stream);
PKV_API int pkv_silu_mul(int32_t dtype, const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride,
                         int64_t rows, int32_t intermediate, pkv_stream_t stream);

/* ------------------------------------------------------------------ metadata builder (GPU) */
/*
 * Decode metadata from a device-resident table mirror, instead of host lists
 * and an H2D copy per step (engine/kv_cache.py:597-609, engine/cuda_graphs.py:64-77):
 * (tables->seq_rows is required; lengths[b] = tokens batch entry b already holds)
 *   positions[b]    = lengths[b]                           (int64, the RoPE position)
 *   slot_mapping[b] = table[p / bs] * bs + p % bs          (int64, the append target)
 *   context_lens[b] = p + 1                                (int32)
 * Rows with seq_rows[b] < 0 are CUDA-graph padding: position 0, slot of the scratch block.
 */
PKV_API int pkv_build_decode_metadata(const pkv_tables* tables, int32_t batch, const int32_t* lengths,
                              int32_t block_size, int32_t scratch_block, int64_t* positions,
                              int64_t* slot_mapping, int32_t* context_lens, int32_t* status_dev,
                              pkv_stream_t stream);

/*
 * Prefill metadata: for sequence s with starts[s] cached tokens and cu_seqlens
 * new ones, write per packed token its position and slot (PagedKVCache.write_index,
 * engine/kv_cache.py:562-573, and the positions of engine/kv_cache.py:262-263).
 */
PKV_API int pkv_build_prefill_metadata(const pkv_tables* tables, int32_t num_seqs, const int32_t* cu_seqlens,
                               const int32_t* starts, int32_t block_size, int64_t total_tokens,
                               int64_t* positions, int64_t* slot_mapping, int32_t* status_dev,
                               pkv_stream_t stream);

/* lengths[seq_rows[b]] += 1 for every b with seq_rows[b] >= 0: PagedDecodeContext.commit
 * (engine/kv_cache.py:622-624) for callers that keep per-slot lengths on the device. */
PKV_API int pkv_commit_decode(const int32_t* seq_rows, int32_t batch, int32_t* lengths, pkv_stream_t stream);

/* Apply (row, column, block) updates to the device table mirror: block_tables[row*stride+col] = block.
 * Mirrors the host allocator's table edits (engine/kv_cache.py:524-526,550). */
PKV_API int pkv_update_tables(int32_t* block_tables, int64_t table_stride, int32_t rows, int32_t cols,
                      const int32_t* updates, int32_t n_updates, int32_t* status_dev, pkv_stream_t stream);

/* Copy whole blocks src[i] -> dst[i], every layer, K and V: copy-on-write of a shared block.
 * The reference never writes a shared block, so it has no counterpart (engine/kv_cache.py:499-501). */
PKV_API int pkv_copy_blocks(const pkv_pool* pool, const int32_t* src, const int32_t* dst, int32_t n,
                    int32_t* status_dev, pkv_stream_t stream);

/* ------------------------------------------------------------------ block manager (host) */
/*
 * The reference's allocator and prefix cache (PagedKVCache host bookkeeping,
 * engine/kv_cache.py:411-560) in C++. Host-only: no CUDA calls.
 * Blocks are handed out least-recently-freed first; a released block keeps its
 * prefix key and goes to the tail, a released block without a key goes to the head;
 * slot ids are taken lowest first and reused last-in first-out.
 */
typedef struct pkv_block_manager pkv_block_manager;

PKV_API int pkv_bm_create(int32_t num_blocks, int32_t block_size, int32_t max_seqs, int32_t max_len,
                  int32_t enable_prefix_caching, pkv_block_manager** out);
PKV_API void pkv_bm_destroy(pkv_block_manager* bm);
/* engine/kv_cache.py:462-464 */
PKV_API int pkv_bm_can_allocate(const pkv_block_manager* bm, int64_t num_tokens, int32_t* out);
/* engine/kv_cache.py:512-529; token_ids may be NULL (n_ids ignored) for no prefix lookup */
PKV_API int pkv_bm_allocate(pkv_block_manager* bm, int64_t num_tokens, const int64_t* token_ids, int64_t n_ids,
                    int32_t* out_slot);
/* engine/kv_cache.py:531-540 */
PKV_API int pkv_bm_register_prefix(pkv_block_manager* bm, int32_t slot, const int64_t* token_ids, int64_t n_ids);
/* engine/kv_cache.py:542-551; *out = 0 when the pool (or max_len) cannot hold num_tokens */
PKV_API int pkv_bm_ensure_capacity(pkv_block_manager* bm, int32_t slot, int64_t num_tokens, int32_t* out);
/* engine/kv_cache.py:553-560; PKV_ERR_DOUBLE_FREE for a slot without a table */
PKV_API int pkv_bm_free(pkv_block_manager* bm, int32_t slot);
/*
 * Positions of the next token of each of n slots (= lengths[slot]), checking that each
 * slot's table holds a block for it: PKV_ERR_OUT_OF_RANGE is the reference's
 * "a sequence has no block for its next token" (engine/kv_cache.py:597-600),
 * PKV_ERR_UNKNOWN_SLOT a slot without a table.
 */
PKV_API int pkv_bm_decode_positions(const pkv_block_manager* bm, const int32_t* slots, int32_t n, int32_t* out);
/*
 * Copy-on-write of shared blocks; no counterpart in the reference, which shares only full
 * blocks no sequence writes again (engine/kv_cache.py:499-501, 536-537), so neither call
 * changes anything on its allocator traces.
 * pkv_bm_fork: a new slot whose table shares every block of src_slot, a partially filled
 * last one included (refcounts + 1; same length). PKV_ERR_NO_BLOCKS without a free slot.
 * pkv_bm_prepare_write: before tokens first_pos .. first_pos + n_tokens - 1 of `slot` are
 * written, each block of that range that another sequence also holds is replaced in this
 * slot's table by a fresh block; (old, fresh) pairs go to `pairs` (2 ints each, at most
 * cap_pairs, else PKV_ERR_WORKSPACE) for pkv_copy_blocks to copy before the write.
 * PKV_ERR_NO_BLOCKS, with nothing changed, when the pool cannot supply them.
 */
PKV_API int pkv_bm_fork(pkv_block_manager* bm, int32_t src_slot, int32_t* out_slot);
PKV_API int pkv_bm_prepare_write(pkv_block_manager* bm, int32_t slot, int64_t first_pos, int64_t n_tokens,
                                 int32_t* pairs, int32_t cap_pairs, int32_t* n_pairs);
/* lengths[slots[i]] += 1 for each i: PagedDecodeContext.commit (engine/kv_cache.py:622-624). */
PKV_API int pkv_bm_commit_decode(pkv_block_manager* bm, const int32_t* slots, int32_t n);
/* lengths[slot] read / write (the reference's public `lengths` dict, engine/kv_cache.py:431) */
PKV_API int pkv_bm_get_length(const pkv_block_manager* bm, int32_t slot, int64_t* out);
PKV_API int pkv_bm_set_length(pkv_block_manager* bm, int32_t slot, int64_t value);
/* the reference's public `block_tables[slot]`: copies up to cap entries, *out_len = table length */
PKV_API int pkv_bm_get_table(const pkv_block_manager* bm, int32_t slot, int32_t* out, int32_t cap, int32_t* out_len);
/* live slots in ascending order */
PKV_API int pkv_bm_live_slots(const pkv_block_manager* bm, int32_t* out, int32_t cap, int32_t* out_len);
PKV_API int pkv_bm_num_free_blocks(const pkv_block_manager* bm, int32_t* out);
PKV_API int pkv_bm_num_free_slots(const pkv_block_manager* bm, int32_t* out);
PKV_API int pkv_bm_prefix_hit_tokens(const pkv_block_manager* bm, int64_t* out);
/* free-pool order (head first), per-block refcounts, and blocks holding a prefix key (ascending) */
PKV_API int pkv_bm_free_order(const pkv_block_manager* bm, int32_t* out, int32_t cap, int32_t* out_len);
PKV_API int pkv_bm_ref_counts(const pkv_block_manager* bm, int32_t* out, int32_t cap);
PKV_API int pkv_bm_cached_blocks(const pkv_block_manager* bm, int32_t* out, int32_t cap, int32_t* out_len);
/* Start (1) or stop (0) recording table edits for pkv_bm_drain_table_edits; off by default. */
PKV_API int pkv_bm_set_journal(pkv_block_manager* bm, int32_t enable);
/*
 * Table edits since the last drain as (slot, column, block) triples, for
 * pkv_update_tables on a device mirror; *out_len = number of triples copied.
 * The journal is cleared by the drain. *overflow = 1 if triples were dropped
 * because cap was too small (the caller should then rebuild its mirror).
 */
PKV_API int pkv_bm_drain_table_edits(pkv_block_manager* bm, int32_t* out, int32_t cap_triples, int32_t* out_len,
                             int32_t* overflow);

/* ------------------------------------------------------------------ scheduler (host) */
/*
 * The reference's continuous-batching Scheduler (engine/scheduler.py:42-169) over a
 * native block manager: the same admission, token-budget, preemption and finish
 * decisions, one call per step. Requests are the caller's sequence ids; the scheduler
 * keeps their tokens (prompt, then outputs) for the prefix lookup at (re)admission.
 * The caller keeps the block manager alive longer than the scheduler; cache calls the
 * engine makes itself (register_prefix, length commits) go to the block manager as before.
 */
typedef struct pkv_scheduler pkv_scheduler;
enum pkv_seq_status { PKV_SEQ_WAITING = 0, PKV_SEQ_RUNNING = 1, PKV_SEQ_FINISHED = 2 };
enum pkv_finish_reason {
  PKV_FINISH_NONE = 0, PKV_FINISH_EOS = 1, PKV_FINISH_LENGTH = 2, PKV_FINISH_MAX_MODEL_LEN = 3, PKV_FINISH_ABORT = 4
};
/* One step's decisions; the caller provides the arrays, `capacity` entries each. */
typedef struct pkv_sched_step {
  int32_t capacity;
  int64_t* prefill_ids;            /* admitted this step, in admission order */
  int32_t* prefill_slots;
  int64_t* prefill_cached_tokens;  /* lengths[slot] after allocate: prefix-cache hit tokens */
  int64_t* decode_ids;             /* running before admission (oldest first): one token each */
  int32_t* decode_slots;
  int64_t* preempted_ids;          /* preempted while making room, in order (now waiting) */
  int32_t n_prefills, n_decodes, n_preempted;
  int64_t* prefill_new_tokens;     /* tokens each prefill processes this step (NULL: not written); the
                                    * rest of the sequence unless chunked prefill splits it */
  int64_t* decode_last_tokens;     /* each decode's last token, the one its step feeds the model: its
                                    * last output, or its last prompt token when a chunked prefill
                                    * left only that one (NULL: not written) */
} pkv_sched_step;

/* static_batching: the reference's scheduling == "static" (nobody joins a running batch) */
PKV_API int pkv_sched_create(pkv_block_manager* bm, int32_t max_num_seqs, int64_t max_num_batched_tokens,
                     int64_t max_model_len, int32_t static_batching, const int64_t* eos_token_ids,
                     int32_t n_eos, pkv_scheduler** out);
PKV_API void pkv_sched_destroy(pkv_scheduler* s);
/* Scheduler.add (engine/scheduler.py:55-64): PKV_ERR_EMPTY_PROMPT / PKV_ERR_PROMPT_TOO_LONG */
PKV_API int pkv_sched_add(pkv_scheduler* s, int64_t seq_id, const int64_t* prompt_ids, int64_t n,
                  int32_t max_tokens, int32_t ignore_eos);
/* Scheduler.schedule (engine/scheduler.py:68-111); PKV_ERR_WORKSPACE if capacity is too small */
PKV_API int pkv_sched_schedule(pkv_scheduler* s, pkv_sched_step* out);
/*
 * Chunked prefill, off by default (the reference has none: README.md:470-473,
 * engine/kv_cache.py:243-249). When on, a prompt is prefilled across steps: each step runs
 * every decode first, then the running sequences still prefilling (oldest first), then
 * admissions from the queue's front, each given what is left of max_num_batched_tokens
 * (prefill_new_tokens says how many); a sequence whose last prompt token is still
 * unwritten decodes it and samples its first token. Admission, allocation and preemption
 * stay the reference's.
 */
PKV_API int pkv_sched_set_chunked_prefill(pkv_scheduler* s, int32_t enable);
/* Scheduler.append_token for n (seq_id, token) pairs in order (engine/scheduler.py:143-159):
 * finish_reasons[i] = PKV_FINISH_*; finished sequences leave running and free their slot. */
PKV_API int pkv_sched_append_tokens(pkv_scheduler* s, const int64_t* seq_ids, const int64_t* tokens, int32_t n,
                            int32_t* finish_reasons);
/* Scheduler.abort (engine/scheduler.py:150-159): *where = PKV_SEQ_WAITING or PKV_SEQ_RUNNING
 * (it was there and is now finished) or PKV_SEQ_FINISHED (already done: nothing happened). */
PKV_API int pkv_sched_abort(pkv_scheduler* s, int64_t seq_id, int32_t* where);
PKV_API int pkv_sched_counts(const pkv_scheduler* s, int32_t* n_waiting, int32_t* n_running,
                     int64_t* num_preemptions);
/* The queues' sequence ids: waiting front first, running oldest first (cap entries each). */
PKV_API int pkv_sched_queues(const pkv_scheduler* s, int64_t* waiting, int64_t* running, int32_t cap);

#ifdef __cplusplus
}
#endif

#endif /* PKV_H_ */
