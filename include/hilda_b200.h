/*
 * hilda_b200.h — C ABI of the B200 (sm_100a) continuous-batching attention path.
 *
 * Every entry point:
 *   - takes plain device pointers, element strides and sizes (no framework types);
 *   - launches on the caller's CUDA stream (`stream` is a cudaStream_t passed as void*);
 *   - performs no allocation and no host synchronisation, so it can be captured in a
 *     CUDA graph (the caller owns every buffer, including workspaces);
 *   - returns HL_OK (0) or a non-zero hl_status; hl_last_error_string() then describes
 *     the failure (thread-local, valid until the next call on the same thread).
 *
 * Memory layouts follow the reference engine (mini_vllm):
 *   - paged KV cache, per layer and per K/V: [num_blocks, block_size, num_kv_heads, head_dim],
 *     row-major, i.e. one "slot" (token) is num_kv_heads*head_dim contiguous elements
 *     (mini_vllm/engine/model_runner.py:196-219);
 *   - slot = block_id * block_size + offset_in_block; slot -1 means "do not store"
 *     (mini_vllm/layers/attention.py:59-80);
 *   - block_tables[b, i] = physical block of the i-th page of sequence b, -1 padded
 *     (mini_vllm/engine/model_runner.py:551-584, 608-612).
 */
#ifndef HILDA_B200_H
#define HILDA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  HL_OK = 0,
  HL_ERR_INVALID = 1,      /* bad argument: shape, stride, alignment, null pointer */
  HL_ERR_CUDA = 2,         /* a CUDA runtime call or kernel launch failed */
  HL_ERR_UNSUPPORTED = 3,  /* a configuration the kernels are not built for */
  HL_ERR_WORKSPACE = 4     /* workspace missing or too small */
} hl_status;

typedef enum {
  HL_KV_BF16 = 0,
  HL_KV_FP8_E4M3 = 1
} hl_kv_dtype;

/* Description of the last error on this thread ("" if none). */
const char* hl_last_error_string(void);

/* Library version, for load checks. */
int hl_version(void);

/* ------------------------------------------------------------------------------------
 * KV store (scatter new K/V rows into the paged cache by slot_mapping).
 * Replaces store_kvcache / store_kvcache_kernel, mini_vllm/layers/attention.py:59-90.
 * key/value: [num_tokens, num_kv_heads, head_dim] bf16 with head stride head_dim and
 * element stride 1 (the reference asserts the same, attention.py:86-89); their row
 * strides (elements between consecutive tokens) may exceed num_kv_heads*head_dim because
 * they are views into the fused qkv projection output.
 * Slots equal to -1 are skipped; slots outside [0, num_slots) are skipped too (the
 * reference kernel would write out of bounds there).
 * ---------------------------------------------------------------------------------- */
int hl_store_kv_bf16(const void* key, const void* value,
                     int64_t key_row_stride, int64_t value_row_stride,
                     void* k_cache, void* v_cache,
                     const int32_t* slot_mapping, int64_t num_tokens, int64_t num_slots,
                     int num_kv_heads, int head_dim, void* stream);

/* FP8 e4m3 store with per-KV-head fp32 scales: cache = sat_e4m3(round_to_nearest_even(x / scale[h])).
 * Replaces store_kvcache_fp8 -> hilda_store_kvcache_fp8, mini_vllm/layers/attention.py:51-52,133
 * (the reference signature has no scales; unit scales reproduce it). */
int hl_store_kv_fp8(const void* key, const void* value,
                    int64_t key_row_stride, int64_t value_row_stride,
                    void* k_cache, void* v_cache,
                    const int32_t* slot_mapping, int64_t num_tokens, int64_t num_slots,
                    int num_kv_heads, int head_dim,
                    const float* k_scale, const float* v_scale, void* stream);

/* Gather BF16 prefill-cache rows at slot_mapping and quantise them into the FP8 decode cache
 * at the same slots, for num_layers layers at once (layer l uses base + l*layer_stride,
 * strides in elements; scales advance by scale_layer_stride floats per layer).
 * Replaces copy_kvcache_fp8 -> hilda_copy_kvcache_fp8, mini_vllm/layers/attention.py:55-56,
 * called per layer by convert_prefill_to_decode_cache, mini_vllm/engine/model_runner.py:484-502. */
int hl_copy_kv_bf16_to_fp8(const void* src_k, const void* src_v, void* dst_k, void* dst_v,
                           const int32_t* slot_mapping, int64_t num_tokens, int64_t num_slots,
                           int num_kv_heads, int head_dim,
                           const float* k_scale, const float* v_scale,
                           int num_layers, int64_t src_layer_stride, int64_t dst_layer_stride,
                           int64_t scale_layer_stride, void* stream);

/* ------------------------------------------------------------------------------------
 * Paged decode attention (one query token per sequence), split-K flash-decoding with an
 * in-kernel last-CTA reduction.
 * Replaces flash_attn_with_kvcache(q.unsqueeze(1), k_cache, v_cache, cache_seqlens=context_lens,
 * block_table=block_tables, softmax_scale, causal=True), mini_vllm/layers/attention.py:162-170,
 * and hilda_paged_attention_fp8_decode, attention.py:134-141 (kv_dtype = HL_KV_FP8_E4M3;
 * k_scale/v_scale may be NULL for unit scales).
 *   q:   [B, Hq, D] bf16, head stride D, row stride q_row_stride (elements)
 *   out: [B, Hq, D] bf16, row stride out_row_stride (elements)
 *   block_tables: [B, bt_stride] int32; only the first max_blocks_per_seq entries are read
 *   context_lens: [B] int32; rows with 0 produce zeros.
 * Requires head_dim == 128, block_size % 256 == 0, Hq % Hk == 0, Hk in {1,2,4,8},
 * Hq/Hk in {1,2,4,8} (FP8) or {1,2,4,8,16} (BF16).  Kernel choice: Hq/Hk >= 4 with batch <= 2048
 * runs the tensor-core kernel of hl_paged_decode_tc (the CUDA-core kernel is issue-bound there);
 * everything else runs the CUDA-core split-K kernel.  The workspace (>= hl_paged_decode_workspace_size bytes) must be
 * zero-filled once before first use; the kernel leaves it ready for the next launch.
 * Launches that share one workspace must not overlap on the GPU.
 * ---------------------------------------------------------------------------------- */
int64_t hl_paged_decode_workspace_size(int batch, int num_q_heads, int head_dim,
                                       int max_blocks_per_seq, int block_size);

int hl_paged_decode(const void* q, int64_t q_row_stride,
                    const void* k_cache, const void* v_cache, int kv_dtype,
                    const float* k_scale, const float* v_scale,
                    const int32_t* block_tables, int64_t bt_stride, int max_blocks_per_seq,
                    const int32_t* context_lens, int batch,
                    int num_q_heads, int num_kv_heads, int head_dim,
                    int block_size, int64_t num_blocks, float softmax_scale,
                    void* out, int64_t out_row_stride,
                    void* workspace, int64_t workspace_bytes, void* stream);

/* The same decode on the tensor cores (no counterpart in the reference): per 128-token tile of
 * one KV head, S^T = K Q^T and O^T = V^T P^T with tcgen05 (M = 128, N = 16: the G <= 16 query
 * heads padded), K/V tiles by TMA, P^T as bf16 hi + lo; one CTA per SM walks an even share of all
 * (sequence, KV head, tile) units and the last CTA of a split (sequence, head) merges the partial
 * results.  FP8 caches: converter warps turn the staged e4m3 tiles into f16 operands (exact) and
 * Q into f16 with an exact power-of-two shift; the products run with f16 operands, P^T as one f16.
 * Same arguments and workspace as hl_paged_decode; needs batch <= 2048, Hq/Hk in {1,2,4,8,16}
 * (BF16) or {1,2,4,8} (FP8), block_size % 128 == 0 (HL_ERR_UNSUPPORTED otherwise).  Measured
 * on B200 at Hq/Hk = 2 it streams the cache slightly below the CUDA-core kernel (0.79 vs 0.82 of
 * HBM peak in the config-2 decode step); at Hq/Hk >= 4 it is the faster one and hl_paged_decode
 * calls it itself.  This entry point forces it for any supported ratio. */
int hl_paged_decode_tc(const void* q, int64_t q_row_stride,
                    const void* k_cache, const void* v_cache, int kv_dtype,
                    const float* k_scale, const float* v_scale,
                    const int32_t* block_tables, int64_t bt_stride, int max_blocks_per_seq,
                    const int32_t* context_lens, int batch,
                    int num_q_heads, int num_kv_heads, int head_dim,
                    int block_size, int64_t num_blocks, float softmax_scale,
                    void* out, int64_t out_row_stride,
                    void* workspace, int64_t workspace_bytes, void* stream);

/* Allocation-free variant of hl_paged_decode (no counterpart in the reference).  For callers
 * that cannot allocate device memory themselves — a host binding this library through an FFI
 * with no device allocator, or a serving loop whose memory is all reserved up front and must not
 * call cudaMalloc (it synchronises the device and can fail under memory pressure) — the split-K
 * scratch is a file-scope device array of hl_paged_decode_noalloc_capacity() bytes (32 MiB),
 * reserved on every GPU that loads the library until the process exits.  Shapes whose
 * hl_paged_decode_workspace_size exceeds it are rejected with HL_ERR_UNSUPPORTED.  The first call
 * on a device looks up the array's device address (make it before any stream capture); each call
 * then clears the array's ticket region on `stream` and launches the same kernel as
 * hl_paged_decode.  All calls share the one array: calls that overlap on the GPU (other streams,
 * other threads) race and must be serialised by the caller.  Allocates nothing. */
int hl_paged_decode_noalloc(const void* q, int64_t q_row_stride,
                            const void* k_cache, const void* v_cache, int kv_dtype,
                            const float* k_scale, const float* v_scale,
                            const int32_t* block_tables, int64_t bt_stride, int max_blocks_per_seq,
                            const int32_t* context_lens, int batch,
                            int num_q_heads, int num_kv_heads, int head_dim,
                            int block_size, int64_t num_blocks, float softmax_scale,
                            void* out, int64_t out_row_stride, void* stream);

/* Size in bytes of the scratch array behind hl_paged_decode_noalloc. */
int64_t hl_paged_decode_noalloc_capacity(void);

/* Error bits (as hl_paged_decode_read_errors) of the most recent hl_paged_decode_noalloc call on
 * the current device: each call clears the word before its launch, so read it after the call
 * whose status matters and before the next one.  Synchronises `stream`; allocates nothing.  Like
 * hl_paged_decode_noalloc it has no counterpart in the reference. */
int hl_paged_decode_noalloc_read_errors(int32_t* errors_out, void* stream);

/* Reads the error word the decode kernel keeps in its workspace (bit 0: an mbarrier wait
 * timed out; bit 1: a block id was out of range).  Synchronous: copies 4 bytes to host. */
int hl_paged_decode_read_errors(const void* workspace, int32_t* errors_out, void* stream);

/* ------------------------------------------------------------------------------------
 * Varlen causal prefill attention (bottom-right aligned causal mask), optionally reading
 * K/V (prefix + chunk) from the paged cache through block_tables, on the 5th-generation tensor
 * cores: tcgen05.mma with TMEM accumulators, Q/K/V tiles brought in by TMA (3-D tensor maps,
 * 128-byte swizzle), S and O resident in TMEM.
 * Replaces flash_attn_varlen_func(q, k|k_cache, v|v_cache, cu_seqlens_q, cu_seqlens_k,
 * max_seqlen_q, max_seqlen_k, softmax_scale, causal=True, block_table),
 * mini_vllm/layers/attention.py:120-131,149-160.
 *   q:   [total_q, Hq, D] bf16 (row stride q_row_stride), out [total_q, Hq, D] (out_row_stride)
 *   paged (block_tables != NULL): k/v are the caches [num_blocks, block_size, Hk, D],
 *   block_size % 128 == 0;
 *   contiguous (block_tables == NULL): k/v are [total_k, Hk, D] with row strides k_row_stride,
 *   v_row_stride, and sequence s's keys are rows cu_seqlens_k[s] .. cu_seqlens_k[s+1]-1.
 * precise_p != 0 feeds the probabilities to the P.V product as two bf16 terms (hi + lo, ~16
 * significant bits; one extra MMA group per tile) instead of one bf16-rounded term, which keeps
 * outputs within an fp32 reference's rtol 2e-2 / atol 2e-3 where heavy cancellation defeats
 * bf16 P (bf16 P alone is what flash-attn does).  Requires head_dim == 128 and Hq % Hk == 0.
 * When Hq / Hk is even, one CTA computes the two query heads of a KV head together (each
 * K/V tile feeds both; P kept in TMEM as the A operand of the P.V MMA); otherwise one head per
 * CTA.  precise_p | HL_PREFILL_ONE_HEAD_PER_CTA forces the one-head kernel (for comparison).
 * ---------------------------------------------------------------------------------- */
#define HL_PREFILL_ONE_HEAD_PER_CTA 2
int hl_varlen_prefill(const void* q, int64_t q_row_stride, int64_t total_q,
                      const void* k, const void* v, int64_t k_row_stride, int64_t v_row_stride,
                      int64_t total_k, const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_k,
                      const int32_t* block_tables, int64_t bt_stride,
                      int num_seqs, int max_seqlen_q,
                      int num_q_heads, int num_kv_heads, int head_dim,
                      int block_size, int64_t num_blocks, float softmax_scale,
                      void* out, int64_t out_row_stride, int precise_p, void* stream);

/* Error bits of the tensor-core prefill kernel (bit 0: an mbarrier wait timed out; bit 1: a
 * block id of a key tile was out of range, the tile read as zeros).  Sticky for the process on
 * the current device.  Synchronous.  Replaces, as a status the host reads, the Python assertions
 * of mini_vllm/layers/attention.py:86-89. */
int hl_varlen_prefill_read_errors(int32_t* errors_out);

/* The same 4 bytes copied asynchronously on `stream` into dst (pinned host or device memory),
 * so a caller can fetch them together with a step's other results without an extra sync. */
int hl_varlen_prefill_copy_errors_async(int32_t* dst, void* stream);

/* Clears the prefill error word (after a caller has handled it); synchronises `stream`. */
int hl_varlen_prefill_clear_errors(void* stream);

/* ------------------------------------------------------------------------------------
 * Decode-batch packing on the GPU.
 * Replaces the host loop of ModelRunner.prepare_decode and its block-table row sync,
 * mini_vllm/engine/model_runner.py:551-584 (_clear_decode_block_table_slot,
 * _copy_decode_block_table_row, _sync_decode_block_table_row) and :652-720.
 * The persistent graph buffers (input_ids int64, positions int64, slot_mapping int32,
 * context_lens int32, block_tables int32 [>= graph_batch rows, bt_stride]) are rebuilt in
 * place from the device's own per-slot state (slot_seq_ids, slot_bt_lens, the previous
 * context_lens) plus a compact host packet of slot events.  A slot in [0, batch) without an
 * event is "continuing": if it has an owner (slot_seq_ids != -1) its context length grows by
 * one and its input id becomes next_tokens[slot] (the token sampled for it in the previous
 * decode step); if it has no owner it is padding.  Slots in [batch, graph_batch) get
 * position 0, context length 0 and slot -1 as the reference pads them
 * (model_runner.py:709-712); their input ids and block-table rows are left as they are.
 *
 * The packet lives in device memory so one launch can be captured in a CUDA graph and
 * replayed with a new packet each step (one host->device copy of the used bytes):
 *   hl_pack_header, then num_events hl_pack_event records, then pool_len int32 block ids
 *   starting at byte pool_offset.  At most one event per slot; graph_batch <= 1024.
 * Out-of-range fields are ignored by the kernel (batch is clamped to graph_batch, events
 * outside the packet or for slots >= batch are skipped, pool reads stay inside the pool).
 * ---------------------------------------------------------------------------------- */
typedef struct {
  int32_t num_events;
  int32_t batch;        /* scheduled decode batch (slots [0, batch) are live or padding) */
  int32_t pool_offset;  /* byte offset of the block-id pool from the start of the packet */
  int32_t pool_len;     /* number of int32 block ids in the pool */
} hl_pack_header;

typedef struct {
  int32_t flags;      /* HL_EV_* bit set */
  int32_t slot;       /* decode slot index, < batch */
  int32_t ctx_len;    /* HL_EV_SCALARS: context length (tokens) of the owning sequence */
  int32_t bt_len;     /* HL_EV_SCALARS / HL_EV_ROW: block-table length after this event */
  int64_t seq_id;     /* HL_EV_SCALARS: id of the owning sequence */
  int64_t token;      /* HL_EV_SCALARS: last token id of the owning sequence */
  int32_t row_start;  /* HL_EV_ROW: first block-table entry written */
  int32_t row_count;  /* HL_EV_ROW: number of entries written from the pool */
  int32_t pool_off;   /* HL_EV_ROW: index of the first entry in the pool */
  int32_t reserved;
} hl_pack_event;

enum {
  HL_EV_SCALARS = 1,   /* slot owned by seq_id with ctx_len tokens, last token `token` */
  HL_EV_ROW = 2,       /* row[row_start : row_start+row_count] := pool[pool_off : ...] */
  HL_EV_ROW_FILL = 4,  /* with HL_EV_ROW: row[row_start+row_count :] := -1 (full rewrite) */
  HL_EV_CLEAR = 8      /* padding slot that had an owner: row := -1, owner and length forgotten */
};

int hl_pack_decode_batch(const void* packet, int64_t packet_bytes, int graph_batch, int block_size,
                         int64_t* slot_seq_ids, int32_t* slot_bt_lens, const int64_t* next_tokens,
                         int64_t* input_ids, int64_t* positions, int32_t* slot_mapping,
                         int32_t* context_lens, int32_t* block_tables, int64_t bt_stride,
                         int max_blocks_per_seq, void* stream);

/* ------------------------------------------------------------------------------------
 * Kernels around attention in the decode/prefill step (bf16 in/out, fp32 arithmetic with
 * the reference's rounding points).
 * ---------------------------------------------------------------------------------- */

/* RMSNorm over `hidden` (multiple of 256, <= 8192).  residual == NULL: out = RMSNorm(in)
 * (mini_vllm/layers/layernorm.py:18-28).  residual != NULL: x = in + residual in fp32,
 * residual := bf16(x), out = RMSNorm(x) (add_rms_forward, layernorm.py:30-42).
 * `residual` rows are contiguous (stride = hidden). */
int hl_rmsnorm(const void* in, int64_t in_stride, void* residual, const void* weight, void* out,
               int64_t out_stride, int rows, int hidden, float eps, void* stream);

/* In place on the fused qkv projection rows [q | k | v]: per-head RMSNorm of q and k with
 * q_weight / k_weight, then NeoX rotary embedding with cos_sin[pos] = [cos | sin] (fp32,
 * head_dim entries per position), positions int64.  head_dim must be 128.
 * Replaces Qwen3Attention.forward's q_norm/k_norm + rotary_emb, mini_vllm/models/qwen3.py:82-85,
 * mini_vllm/layers/rotary_embedding.py:8-16,39-50. */
int hl_qk_norm_rope(void* qkv, int64_t row_stride, int num_tokens, int num_q_heads, int num_kv_heads,
                    int head_dim, const void* q_weight, const void* k_weight, const float* cos_sin,
                    const int64_t* positions, float eps, void* stream);

/* hl_qk_norm_rope fused with the KV-cache store: after rotating row t in place, writes the
 * post-RoPE k heads and the v heads of row t to row slot_mapping[t] of k_cache / v_cache
 * ([num_slots, Hk*D], kv_dtype HL_KV_BF16 or HL_KV_FP8_E4M3 with optional per-head scales),
 * skipping slots outside [0, num_slots).  Replaces the qwen3.py:82-85 prologue plus the
 * store_kvcache / store_kvcache_fp8 calls at mini_vllm/layers/attention.py:133,146 in one
 * launch; the cache bytes equal those of hl_store_kv_bf16 / hl_store_kv_fp8 applied to the
 * rotated rows.  k_cache = v_cache = NULL makes it exactly hl_qk_norm_rope. */
int hl_qk_norm_rope_store(void* qkv, int64_t row_stride, int num_tokens, int num_q_heads, int num_kv_heads,
                          int head_dim, const void* q_weight, const void* k_weight, const float* cos_sin,
                          const int64_t* positions, float eps, void* k_cache, void* v_cache, int kv_dtype,
                          const int32_t* slot_mapping, int64_t num_slots, const float* k_scale,
                          const float* v_scale, void* stream);

/* hl_qk_norm_rope_store with an FP8 store (kv_dtype = HL_KV_FP8_E4M3) that also writes the
 * rotated bf16 K rows and the V rows into k_mirror / v_mirror (bf16 caches of the same
 * [num_slots, Hk*128] row layout): the FP8 mode's BF16 prefill cache then holds the decode-step
 * tokens as well.  The reference's decode step writes only the FP8 cache
 * (mini_vllm/layers/attention.py:133), so a prefix-cache hit on a block filled during decode
 * (block_manager.py may_append registers it) followed by the prefill->decode copy
 * (model_runner.py:484-502) reads stale BF16 rows; with the mirror both caches agree.
 * k_mirror = v_mirror = NULL makes it exactly hl_qk_norm_rope_store. */
int hl_qk_norm_rope_store_mirrored(void* qkv, int64_t row_stride, int num_tokens, int num_q_heads,
                                   int num_kv_heads, int head_dim, const void* q_weight, const void* k_weight,
                                   const float* cos_sin, const int64_t* positions, float eps, void* k_cache,
                                   void* v_cache, int kv_dtype, const int32_t* slot_mapping, int64_t num_slots,
                                   const float* k_scale, const float* v_scale, void* k_mirror, void* v_mirror,
                                   void* stream);

/* out = silu(in[:, :I]) * in[:, I:2I]  (SiluAndMul, mini_vllm/layers/activation.py:12-16). */
int hl_silu_mul(const void* in, int64_t in_stride, void* out, int64_t out_stride, int rows,
                int intermediate, void* stream);

/* Greedy token per row: argmax over bf16 logits, lowest index among equal maxima
 * (the greedy replacement of Sampler.forward, mini_vllm/layers/sampler.py:12-25). */
int hl_argmax(const void* logits, int64_t row_stride, int rows, int vocab, int64_t* out_tokens,
              void* stream);

/* Greedy token of one vocabulary shard under tensor parallelism: per row the index of the
 * maximum plus index_offset (the shard's first vocabulary id) and the maximum itself, so ranks
 * can all-gather (value, index) pairs instead of the logits that the reference gathers to rank 0
 * (mini_vllm/layers/embed_head.py:56-66). */
int hl_argmax_shard(const void* logits, int64_t row_stride, int rows, int vocab, int64_t index_offset,
                    int64_t* out_tokens, float* out_values, void* stream);

/* ------------------------------------------------------------------------------------
 * Tensor-parallel all-reduce over NVLink peer memory fused with add + RMSNorm.
 * Replaces dist.all_reduce after o_proj / down_proj (mini_vllm/layers/linear.py:176-178)
 * together with the add + RMSNorm that follows it (layers/layernorm.py:30-42).
 * Each rank allocates its partial-sum buffers and a signal area (hl_device_alloc, zeroed),
 * shares them with hl_ipc_get_handle / hl_ipc_open_handle, and then, on every rank, with
 * the same rows and the same order of calls:
 *   x = bf16(sum over ranks p in order 0..world-1 of peer_data[p][row, :])   (fp32 sum)
 *   x = x + residual (fp32); residual := bf16(x); out = bf16(bf16(x * rsqrt(mean(x^2)+eps)) * w)
 * peer_data / peer_signal are host arrays of world device pointers (this rank's own at index
 * rank); signal areas hold hl_allreduce_signal_bytes() bytes; epochs is this rank's int32
 * [128] call counter array (zeroed), error_word this rank's int32.  hidden % 256 == 0, <= 8192.
 * Partial-sum buffers must alternate between consecutive calls (two buffers), which makes one
 * barrier per call sufficient.  A peer that does not arrive within timeout_ns sets
 * HL_AR_TIMEOUT in *error_word and the call treats the partial sums as zero instead of hanging.
 * ---------------------------------------------------------------------------------- */
#define HL_AR_TIMEOUT 1

int hl_device_alloc(int64_t bytes, void** ptr_out);
int hl_device_free(void* ptr);
/* cudaIpcMemHandle_t is 64 bytes. */
int hl_ipc_get_handle(void* dev_ptr, void* handle_out);
int hl_ipc_open_handle(const void* handle, void** dev_ptr_out);
int hl_ipc_close_handle(void* dev_ptr);
int64_t hl_allreduce_signal_bytes(void);
int hl_allreduce_add_rmsnorm(void* const* peer_data, void* const* peer_signal, int world, int rank,
                             int rows, int hidden, void* residual, const void* weight, void* out,
                             int64_t out_stride, float eps, int* epochs, int* error_word,
                             int64_t timeout_ns, void* stream);

/* Two-shot form of hl_allreduce_add_rmsnorm for more than two ranks, same result bit for bit:
 * rank p sums only rows r with r % world == p (reading them from every rank) and stores the bf16
 * sum into every rank's result buffer (peer_result: world device pointers to [rows, hidden] bf16
 * buffers, mapped like peer_data); after a second barrier every rank applies the add + RMSNorm
 * to all rows from its own result buffer.  Per call each rank moves 2 (world - 1) / world of the
 * rows over NVLink instead of (world - 1) x the rows.  rows <= 512; signal areas as above (the
 * second barrier uses their second half).  Replaces the same calls as hl_allreduce_add_rmsnorm
 * (mini_vllm/layers/linear.py:176-178 with layers/layernorm.py:30-42). */
int hl_allreduce_add_rmsnorm_2shot(void* const* peer_data, void* const* peer_result, void* const* peer_signal,
                                   int world, int rank, int rows, int hidden, void* residual,
                                   const void* weight, void* out, int64_t out_stride, float eps, int* epochs,
                                   int* error_word, int64_t timeout_ns, void* stream);

/* Token per row of bf16 logits: rows with temperatures[row] > 0 are sampled by the Gumbel-max
 * trick, argmax_i (logit_i / T + Gumbel noise) — the distribution of the reference's
 * exponential-race Sampler with top_k = -1, top_p = 1 (mini_vllm/layers/sampler.py:12-25) — the
 * others (or all, temperatures = NULL) take the greedy argmax.  The noise is a counter-based hash
 * of (seed, step, row, index_offset + i), so vocabulary shards of a tensor-parallel LM head draw
 * disjoint parts of the same noise; out_values (optional) receives the winning perturbed value for
 * merging shards.  step_state: device uint64[2] (zeroed once); the launch reads the step and its
 * last row advances it, so CUDA-graph replays draw fresh noise.  NULL: step 0 every call. */
int hl_sample(const void* logits, int64_t row_stride, int rows, int vocab, int64_t index_offset,
              const float* temperatures, uint64_t seed, void* step_state, int64_t* out_tokens,
              float* out_values, void* stream);

/* hl_sample with the reference's top-k and top-p filters (mini_vllm/layers/sampler.py:13-49):
 * per row x = logit / T; top_ks[row] in (0, vocab) keeps the k largest x; top_ps[row] < 1 then
 * keeps, in descending order of x, the tokens whose inclusive cumulative softmax probability over
 * the top-k set is below top_p (always at least the first); the token is the Gumbel-max draw over
 * what is kept, with hl_sample's noise, so a row without filters gets exactly hl_sample's token.
 * Where a filter boundary cuts through equal logits, lower vocabulary ids come first (torch.sort
 * leaves that order unspecified).  top_ks / top_ps may be NULL (no filter); rows with T <= 0 take
 * the greedy argmax.  Full-vocabulary rows only (no index_offset: vocabulary shards of a
 * tensor-parallel head cannot decide a global top-k).  step_state as for hl_sample. */
int hl_sample_filtered(const void* logits, int64_t row_stride, int rows, int vocab,
                       const float* temperatures, const int32_t* top_ks, const float* top_ps,
                       uint64_t seed, void* step_state, int64_t* out_tokens, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HILDA_B200_H */
