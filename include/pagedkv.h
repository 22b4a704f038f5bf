/*
 * pagedkv.h -- C ABI of libpagedkv.so, the B200 (sm_100a) paged-KV-cache hot
 * path for mini_engine (kjoshiDTX/llm-inference-scheduler).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as an opaque pointer so this header needs no CUDA include), is
 * asynchronous with respect to the host, allocates nothing, and returns an
 * int status: 0 = ok, < 0 = an argument error detected on the host before
 * anything was launched (see PKV_ERR_*), > 0 = the cudaError_t reported by
 * the launch.  Kernels never trap: an out-of-range block id, slot or context
 * length found on the device is skipped or clamped and recorded with atomicOr
 * into *err_flags (PKV_FLAG_*), when err_flags is not NULL.
 *
 * Layouts (the reference's, block_manager.py:10-13,37):
 *   pool      [num_blocks][block_size][n_kv_heads][head_dim], one per layer
 *   q, out    [n_tokens][n_q_heads][head_dim] with a row stride in elements
 *   k, v new  [n_tokens][n_kv_heads][head_dim] with a row stride in elements
 *   slot      block * block_size + offset (int64), -1 = padding, skipped
 *   tables    [n_seqs][block_table_stride] int32 physical block ids
 *
 * Threading: calls may come from any host thread; the library keeps only a
 * mutex-protected cache of TMA descriptors.  One call = one or two kernel
 * launches on `stream`.
 */
#ifndef PAGEDKV_H
#define PAGEDKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PKV_ABI_VERSION 1

/* element types of q / k / v / pools / out */
#define PKV_DTYPE_F32 0
#define PKV_DTYPE_F16 1
#define PKV_DTYPE_BF16 2

/* host-side status codes */
#define PKV_OK 0
#define PKV_ERR_NULL_POINTER (-1)
#define PKV_ERR_BAD_SHAPE (-2)
#define PKV_ERR_BAD_DTYPE (-3)
#define PKV_ERR_WORKSPACE_TOO_SMALL (-4)
#define PKV_ERR_MISALIGNED (-5)
#define PKV_ERR_UNSUPPORTED (-6)
#define PKV_ERR_DRIVER (-7)
#define PKV_ERR_SCRATCH_LIMIT (-8)

/* device-side error flag bits (atomicOr into *err_flags) */
#define PKV_FLAG_SLOT_OUT_OF_RANGE 1
#define PKV_FLAG_BLOCK_OUT_OF_RANGE 2
#define PKV_FLAG_CONTEXT_EXCEEDS_TABLE 4
#define PKV_FLAG_PIPELINE_TIMEOUT 8
#define PKV_FLAG_BAD_QUERY_LAYOUT 16
#define PKV_FLAG_POSITION_OUT_OF_RANGE 32
#define PKV_FLAG_BAD_SCHEDULE 64 /* a decode schedule built for another batch, grid or table width */

/* size of the device-resident scratch array behind
 * pkv_paged_decode_attention_noalloc (per GPU, held until the process exits) */
#define PKV_NOALLOC_SCRATCH_BYTES (8u << 20)

/* Bytes of a CUDA IPC memory handle (pkv_ipc_export / pkv_ipc_open). */
#define PKV_IPC_HANDLE_BYTES 64

/* decode-attention kernel choice (pkv_set_decode_impl) */
/* flags of pkv_paged_decode_append_attention_layers_flags */
#define PKV_LAYERS_DEFER_FIRST 1

#define PKV_DECODE_AUTO 0
#define PKV_DECODE_GENERIC 1

typedef void* pkv_stream_t; /* a cudaStream_t; NULL = legacy default stream */

/* ABI version of the loaded library (PKV_ABI_VERSION it was built with). */
int pkv_abi_version(void);

/* Static description of a status code or error-flag word; never NULL. */
const char* pkv_status_string(int status);

/*
 * KV append.  Replaces the scatter loop of PagedKVCache.append_and_fetch
 * (mini_engine/paged/block_manager.py:121-131): token t's K and V rows are
 * written to pool row slot_mapping[t]; slot -1 is skipped (padding).  One
 * launch per layer covers every sequence of the step.  Bit-exact copy.
 * A slot >= num_blocks * block_size sets PKV_FLAG_SLOT_OUT_OF_RANGE and is
 * skipped.
 */
int pkv_reshape_and_cache(const void* k, const void* v, int64_t k_row_stride,
                          int64_t v_row_stride, void* k_pool, void* v_pool,
                          const int64_t* slot_mapping, int n_tokens, int num_blocks,
                          int block_size, int n_kv_heads, int head_dim, int dtype,
                          int* err_flags, pkv_stream_t stream);

/*
 * Copy-on-write / fork block copies.  Replaces BlockManager.copy_block's
 * per-layer loop (mini_engine/paged/block_manager.py:65-71), batched: for each
 * (src, dst) pair in block_pairs [n_pairs][2] and each of n_layers layers,
 * the K and V block dst becomes a copy of block src.  Layer l's pool starts
 * at k_pools + l * layer_stride_bytes (same for v_pools).  dst blocks must
 * be distinct and must not appear as a src in the same call.  An id outside
 * [0, num_blocks) sets PKV_FLAG_BLOCK_OUT_OF_RANGE and the pair is skipped.
 */
int pkv_copy_blocks(void* k_pools, void* v_pools, int64_t layer_stride_bytes, int n_layers,
                    const int32_t* block_pairs, int n_pairs, int num_blocks,
                    int64_t block_bytes, int* err_flags, pkv_stream_t stream);

/*
 * The fp8 decode step of one layer in one launch: each sequence's new K/V
 * token (k_new / v_new rows in `dtype`) is quantised into the fp8 pools at
 * position context_lens[s] - 1 (as pkv_reshape_and_cache_fp8 quantises it,
 * with its scales) by the decode kernel itself, then the fp8 decode
 * attention runs (pkv_paged_decode_attention_fp8 semantics).  Replaces, for
 * fp8 pools, the scatter of PagedKVCache.append_and_fetch
 * (mini_engine/paged/block_manager.py:121-131) plus the decode attention.
 */
int pkv_paged_decode_append_attention_fp8(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_new,
    const void* v_new, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pool,
    void* v_pool, float* k_scale, float* v_scale, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream);
int pkv_paged_decode_append_attention_fp8_scheduled(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_new,
    const void* v_new, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pool,
    void* v_pool, float* k_scale, float* v_scale, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule);

/*
 * pkv_paged_decode_append_attention_layers for fp8 e4m3 pools: for layer
 * l = 0 .. n_layers-1 exactly pkv_paged_decode_append_attention_fp8(_scheduled)
 * with the per-layer pointers advanced by their layer strides, the scale
 * arrays by scale_layer_stride floats ([num_layers][num_blocks][block_size]
 * [Hkv] scales).  A workspace of n_layers x pkv_decode_workspace_bytes
 * chains the layers on the tensor-core path as in the 16-bit call (each later
 * decode starts on the SMs the previous one's tail frees, one merge launch for
 * every layer); with a single set each layer's decode has its own merge.
 * dtype: the q / out / new-row type (PKV_DTYPE_F16 or PKV_DTYPE_BF16).
 * Replaces, for fp8 pools, the per-layer loop of Qwen2Model.forward
 * (mini_engine/model/qwen2.py:159-166) over append_and_fetch + _attention.
 */
int pkv_paged_decode_append_attention_fp8_layers(
    int n_layers, void* out, int64_t out_layer_stride, int64_t out_row_stride, const void* q,
    int64_t q_layer_stride, int64_t q_row_stride, const void* k_new, const void* v_new,
    int64_t new_layer_stride, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pools,
    void* v_pools, int64_t pool_layer_stride_bytes, float* k_scales, float* v_scales,
    int64_t scale_layer_stride, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule);

/*
 * Chunked prefill over fp8 e4m3 pools on the tensor cores with no scratch:
 * the tcgen05 prefill kernel stages each key tile's e4m3 bytes and row
 * scales in shared memory, and two of its warps convert them into the fp16
 * tiles its MMAs read (value x scale as an fp32 product rounded once to
 * fp16, as the scratch pass rounds it), so no pass over the visible blocks writes a 16-bit copy
 * to memory.  Same arguments and semantics as pkv_paged_prefill_attention_fp8
 * (which stays the CUDA-core kernel).  Serves fp16 queries (dtype
 * PKV_DTYPE_F16), head_dim 64, block_size 16, up to 4 KV heads, 16-byte
 * aligned pools and scale arrays; other cases return PKV_ERR_UNSUPPORTED.
 * For callers that cannot hold the scratch: every CTA converts the tiles it
 * reads, where the scratch pass converts each visible block once, so at
 * config 4's shape this entry is about a quarter slower than
 * pkv_paged_prefill_attention_fp8_scratch.  Replaces, for fp8 pools, the
 * gather + _attention of mini_engine/model/qwen2.py:98-128 with num_new > 1.
 */
int pkv_paged_prefill_attention_fp8_tc(void* out, int64_t out_row_stride, const void* q,
                                       int64_t q_row_stride, const void* k_pool, const void* v_pool,
                                       const float* k_scale, const float* v_scale, int num_blocks,
                                       const int32_t* block_tables, int64_t block_table_stride,
                                       int max_blocks_per_seq, const int32_t* query_start_loc,
                                       const int32_t* num_prior, int n_seqs, int n_tokens,
                                       int max_query_len, int n_q_heads, int n_kv_heads,
                                       int head_dim, int block_size, float scale, int dtype,
                                       int* err_flags, pkv_stream_t stream);

/*
 * Chunked prefill over fp8 e4m3 pools on the tensor cores.  Same arguments
 * and semantics as pkv_paged_prefill_attention_fp8, plus a caller-provided
 * scratch buffer (pkv_prefill_fp8_scratch_bytes(n_seqs, max_blocks_per_seq,
 * n_kv_heads, head_dim) bytes, 256-byte aligned, any contents): one pass
 * writes the blocks the step can see there as 16-bit rows (e4m3 x scale,
 * rounded once to `dtype`), then the tcgen05 prefill kernel runs over them.
 * The results differ from the CUDA-core fp8 prefill by that one rounding.
 * Shapes the tensor-core kernel does not serve fall back to the CUDA-core
 * kernel (the scratch is then unused).  Replaces, for fp8 pools, the gather
 * and _attention with num_new > 1 (mini_engine/paged/block_manager.py:136-141,
 * mini_engine/model/qwen2.py:98-128).
 */
size_t pkv_prefill_fp8_scratch_bytes(int n_seqs, int max_blocks_per_seq, int n_kv_heads,
                                     int head_dim);
int pkv_paged_prefill_attention_fp8_scratch(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_pool,
    const void* v_pool, const float* k_scale, const float* v_scale, int num_blocks,
    const int32_t* block_tables, int64_t block_table_stride, int max_blocks_per_seq,
    const int32_t* query_start_loc, const int32_t* num_prior, int n_seqs, int n_tokens,
    int max_query_len, int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale,
    int dtype, void* scratch, size_t scratch_bytes, int* err_flags, pkv_stream_t stream);

/*
 * Per-step decode schedule.  All layers of a decode step share the block
 * tables and context lengths, so the stream-K partition of the step's blocks
 * over the decode kernel's persistent CTAs is the same for every layer.
 * pkv_decode_schedule computes it once per step (one small kernel: clamped
 * lengths, block prefix, each CTA's block ids, with the bounds checks and
 * their error flags), and the _scheduled decode calls read it instead of
 * recomputing it in every layer's prologue.  The schedule buffer is
 * caller-provided (pkv_decode_schedule_bytes, 16-byte aligned); n_q_heads,
 * n_kv_heads, head_dim, block_size, dtype and fp8_pools (1 for the fp8
 * decode) must be those of the decode calls that use it, and block_tables /
 * context_lens must not change between building and using it.  A schedule
 * built for another batch size, grid or max_blocks_per_seq (table width)
 * sets PKV_FLAG_BAD_SCHEDULE and the decode call reads nothing of it and
 * does nothing.  Shapes the tensor-core decode kernel does not serve
 * build nothing and their _scheduled calls ignore the schedule.  The first
 * decode launch after a build is stream-ordered behind it.
 */
size_t pkv_decode_schedule_bytes(int n_seqs, int max_blocks_per_seq);
int pkv_decode_schedule(void* schedule, size_t schedule_bytes, const int32_t* block_tables,
                        int64_t block_table_stride, int max_blocks_per_seq,
                        const int32_t* context_lens, int n_seqs, int num_blocks, int n_q_heads,
                        int n_kv_heads, int head_dim, int block_size, int dtype, int fp8_pools,
                        int* err_flags, pkv_stream_t stream);
/* pkv_paged_decode_attention / _fp8 / _append_attention with a schedule
 * (the same arguments, then the schedule) */
int pkv_paged_decode_attention_scheduled(void* out, int64_t out_row_stride, const void* q,
                                         int64_t q_row_stride, const void* k_pool,
                                         const void* v_pool, int num_blocks,
                                         const int32_t* block_tables, int64_t block_table_stride,
                                         int max_blocks_per_seq, const int32_t* context_lens,
                                         int n_seqs, int n_q_heads, int n_kv_heads, int head_dim,
                                         int block_size, float scale, int dtype, void* workspace,
                                         size_t workspace_bytes, int* err_flags,
                                         pkv_stream_t stream, const void* schedule);
int pkv_paged_decode_attention_fp8_scheduled(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_pool,
    const void* v_pool, const float* k_scale, const float* v_scale, int num_blocks,
    const int32_t* block_tables, int64_t block_table_stride, int max_blocks_per_seq,
    const int32_t* context_lens, int n_seqs, int n_q_heads, int n_kv_heads, int head_dim,
    int block_size, float scale, int dtype, void* workspace, size_t workspace_bytes,
    int* err_flags, pkv_stream_t stream, const void* schedule);
int pkv_paged_decode_append_attention_scheduled(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_new,
    const void* v_new, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pool,
    void* v_pool, int num_blocks, const int32_t* block_tables, int64_t block_table_stride,
    int max_blocks_per_seq, const int32_t* context_lens, int n_seqs, int n_q_heads,
    int n_kv_heads, int head_dim, int block_size, float scale, int dtype, void* workspace,
    size_t workspace_bytes, int* err_flags, pkv_stream_t stream, const void* schedule);

/*
 * A decode step over a run of consecutive layers in one call: for layer
 * l = 0 .. n_layers-1 exactly pkv_paged_decode_append_attention(_scheduled)
 * with every per-layer pointer advanced by l times its layer stride.  Replaces
 * the per-layer loop of Qwen2Model.forward (mini_engine/model/qwen2.py:
 * 159-166) over PagedKVCache.append_and_fetch (block_manager.py:111-141) +
 * _attention, for a step whose sequences all decode one token and whose
 * layers' q / k / v are ready together (e.g. copied in from the host at
 * once): one host call issues 2 x n_layers launches instead of n_layers
 * calls, each with its own argument checks.
 *   q, out       : layer l at + l * q_layer_stride / out_layer_stride elements;
 *   k_new, v_new : layer l at + l * new_layer_stride elements;
 *   k_pools, v_pools : layer l's pool at + l * pool_layer_stride_bytes bytes
 *                  (the [num_layers][num_blocks][block_size][Hkv][D] caches).
 * Tables, lengths, scale and schedule are shared by the layers (a schedule
 * built for the step serves them all; NULL: none).  Workspace: with
 * workspace_bytes >= n_layers x pkv_decode_workspace_bytes (one split-K set
 * per layer, layer l's at l x that size), the layers chain on the
 * tensor-core path: each later layer's decode kernel starts on the SMs the
 * previous layer's tail frees (it waits for its predecessor only at its
 * end; nothing it reads is written by the layers before it), and one merge
 * launch after the last decode covers every layer.  With a single set, every
 * layer's decode is followed by its own merge.  The results are the same
 * bits either way.  Arguments
 * are checked for the first and the last layer before anything launches; on
 * a launch error the call returns it and the later layers are not issued.
 * input_ready: NULL, or n_layers 4-byte aligned device words.  Layer l's
 * decode kernel waits until input_ready[l] is nonzero before it reads layer
 * l's q, k_new or v_new; the wait is bounded (about a second): on a timeout
 * it sets PKV_FLAG_PIPELINE_TIMEOUT and the call's outputs are unspecified.
 * It is for inputs that a copy on another stream brings in: the copy stream
 * sets a layer's word after that layer's rows (a 4-byte copy from a host
 * word holding 1, the words cleared before the data copies), and the call
 * needs no event wait on that stream.  Such a wait between two launches of
 * the chain would end their programmatic overlap (about 5 us per chain
 * break on B200).  Only the tensor-core
 * decode kernel serves it: other shapes return PKV_ERR_UNSUPPORTED.
 */
int pkv_paged_decode_append_attention_layers(
    int n_layers, void* out, int64_t out_layer_stride, int64_t out_row_stride, const void* q,
    int64_t q_layer_stride, int64_t q_row_stride, const void* k_new, const void* v_new,
    int64_t new_layer_stride, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pools,
    void* v_pools, int64_t pool_layer_stride_bytes, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule, const int32_t* input_ready);

/*
 * pkv_paged_decode_append_attention_layers with flags (0: the same call).
 * PKV_LAYERS_DEFER_FIRST: the call's first decode kernel also starts before
 * the launch before it completes and waits for it only at its end, as the
 * call's later layers do, so two calls over consecutive runs of layers form
 * one chain: the next run's first layer starts while the previous run's
 * merge is still running, instead of after it.  With the flag the caller
 * promises that no work enqueued before the call and possibly still running
 * writes anything the call reads (the q / k_new / v_new rows, the pools,
 * tables, lengths, schedule) or reads or writes anything it writes (out, the
 * pools' appended slots, the workspace): in particular the previous run used
 * other split-K sets, which is why a step's runs take slices of one
 * workspace of a set per layer of the step.  Inputs still arriving from a
 * copy stream are covered by input_ready.  The flag needs the chained form
 * (a split-K set per layer of the call, a single layer included); otherwise
 * it is ignored and the call runs as without it.  Other flag bits return
 * PKV_ERR_UNSUPPORTED.
 */
int pkv_paged_decode_append_attention_layers_flags(
    int n_layers, void* out, int64_t out_layer_stride, int64_t out_row_stride, const void* q,
    int64_t q_layer_stride, int64_t q_row_stride, const void* k_new, const void* v_new,
    int64_t new_layer_stride, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pools,
    void* v_pools, int64_t pool_layer_stride_bytes, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule, const int32_t* input_ready, int flags);

/*
 * KV block migration between GPUs (one process per GPU).  Replaces the
 * reference's recompute preemption (mini_engine/scheduler.py:143-156 frees a
 * preempted sequence's blocks and recomputes its KV later): a rank copies a
 * sequence's blocks into another rank's pool over NVLink instead.
 *
 * pkv_ipc_export: the CUDA IPC handle (PKV_IPC_HANDLE_BYTES) of the device
 *   allocation that holds dev_ptr, and dev_ptr's byte offset in it (a pool
 *   tensor may sit inside a larger allocation of the caller's allocator).
 * pkv_ipc_open: maps an allocation exported by another process (any GPU of
 *   this node; peer access is enabled on first use) into this process's
 *   current device context and returns its base; add the exported offset.
 *   An allocation is opened once per process.
 * pkv_ipc_close: unmaps a base returned by pkv_ipc_open.
 * pkv_copy_blocks_peer: for each (src, dst) pair of block_pairs [n_pairs][2]
 *   and each of n_layers layers, block dst of the destination K and V pools
 *   becomes a copy of block src of the source pools.  Either side may be a
 *   peer GPU's memory opened with pkv_ipc_open (the kernel runs on the
 *   caller's stream and device).  Layer l of a pool starts l * its layer
 *   stride after its base.  Ids outside [0, num_blocks) of their pool set
 *   PKV_FLAG_BLOCK_OUT_OF_RANGE and the pair is skipped.  block_bytes,
 *   strides and pool bases must be multiples of 16 bytes.  fp8 pools move
 *   their scale pools by a second call (block_bytes = block_size x n_kv_heads
 *   x 4).  The caller orders the copy against the other process's use of
 *   its pool (pagedkv.migration does it with host messages).
 */
int pkv_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset);
int pkv_ipc_open(const void* handle, void** base);
int pkv_ipc_close(void* base);
int pkv_copy_blocks_peer(void* dst_k, void* dst_v, int64_t dst_layer_stride_bytes,
                         int dst_num_blocks, const void* src_k, const void* src_v,
                         int64_t src_layer_stride_bytes, int src_num_blocks, int n_layers,
                         const int32_t* block_pairs, int n_pairs, int64_t block_bytes,
                         int* err_flags, pkv_stream_t stream);

/*
 * Rotary embedding of q and k fused with the KV append (one launch per
 * layer).  Replaces the RoPE of the projected q and k in Qwen2Model.forward
 * (mini_engine/model/qwen2.py:152-158; K is cached post-RoPE) followed by the
 * scatter of PagedKVCache.append_and_fetch (block_manager.py:121-131).
 *   qkv[t]  : one row per token, [q heads | k heads | v heads] x head_dim
 *             (the fused q/k/v projection), qkv_row_stride elements apart;
 *   q_out[t]: the rotated q, [n_q_heads][head_dim], q_out_row_stride apart;
 *   k_pool / v_pool at slot_mapping[t] (as pkv_reshape_and_cache): the
 *             rotated k and the unrotated v.
 * Rotation of the half-split pairs (i, i + head_dim/2) with the caller's
 * tables cos_table / sin_table [max_position][head_dim] (the model dtype),
 * row positions[t]; each product and the sum are rounded to the element type
 * as separate elementwise multiply and add operations round them, so the
 * result equals that unfused computation bit for bit.  A position outside
 * [0, max_position) sets PKV_FLAG_POSITION_OUT_OF_RANGE and the token is
 * skipped; slot -1 writes only q; a slot past the pool sets
 * PKV_FLAG_SLOT_OUT_OF_RANGE.  head_dim must be even.
 */
int pkv_rope_reshape_and_cache(void* q_out, int64_t q_out_row_stride, const void* qkv,
                               int64_t qkv_row_stride, const int64_t* positions,
                               const void* cos_table, const void* sin_table, int max_position,
                               void* k_pool, void* v_pool, const int64_t* slot_mapping,
                               int n_tokens, int num_blocks, int block_size, int n_q_heads,
                               int n_kv_heads, int head_dim, int dtype, int* err_flags,
                               pkv_stream_t stream);
/* The same for fp8 e4m3 pools (uint8 k_pool / v_pool): the rotated k and the
 * v rows are quantised as pkv_reshape_and_cache_fp8 quantises them (one fp32
 * scale per (slot, KV head) into k_scale / v_scale), bit-identical to rotating
 * in `dtype` and calling it.  q_out stays in `dtype`. */
int pkv_rope_reshape_and_cache_fp8(void* q_out, int64_t q_out_row_stride, const void* qkv,
                                   int64_t qkv_row_stride, const int64_t* positions,
                                   const void* cos_table, const void* sin_table, int max_position,
                                   void* k_pool, void* v_pool, float* k_scale, float* v_scale,
                                   const int64_t* slot_mapping, int n_tokens, int num_blocks,
                                   int block_size, int n_q_heads, int n_kv_heads, int head_dim,
                                   int dtype, int* err_flags, pkv_stream_t stream);

/*
 * Bytes of device workspace pkv_paged_decode_attention needs for n_seqs
 * sequences (split-K partials; no initialisation required).
 */
size_t pkv_decode_workspace_bytes(int n_seqs, int n_q_heads, int head_dim);

/*
 * Paged decode attention (one new query token per sequence).  Replaces the
 * gather of PagedKVCache.append_and_fetch (block_manager.py:136-141) plus
 * Qwen2Model._attention with num_new == 1 (mini_engine/model/qwen2.py:98-128):
 *   out[s, h, :] = softmax_j(scale * q[s, h, :] . K_s[j, h / G, :]) V_s[j, h / G, :]
 * over the context_lens[s] tokens of sequence s, read in place through
 * block_tables[s] (G = n_q_heads / n_kv_heads).  The new token must already
 * have been written (pkv_reshape_and_cache).  context_lens[s] == 0 gives a
 * zero row.  `workspace` (pkv_decode_workspace_bytes) carries split-K
 * partials from the decode kernel to the merge kernel of the same call; calls
 * that may overlap on the GPU need separate workspaces.
 */
int pkv_paged_decode_attention(void* out, int64_t out_row_stride, const void* q,
                               int64_t q_row_stride, const void* k_pool, const void* v_pool,
                               int num_blocks, const int32_t* block_tables,
                               int64_t block_table_stride, int max_blocks_per_seq,
                               const int32_t* context_lens, int n_seqs, int n_q_heads,
                               int n_kv_heads, int head_dim, int block_size, float scale,
                               int dtype, void* workspace, size_t workspace_bytes,
                               int* err_flags, pkv_stream_t stream);

/*
 * Decode step of one layer in one call: append + paged decode attention.
 * Replaces PagedKVCache.append_and_fetch (block_manager.py:111-141: scatter,
 * length update, gather) followed by Qwen2Model._attention with num_new == 1
 * (qwen2.py:98-128).  For every sequence s with context_lens[s] >= 1, the
 * new token's K and V rows (k_new[s], v_new[s]: [n_seqs][n_kv_heads][head_dim]
 * with the given row strides) are written to position context_lens[s] - 1 of
 * the sequence, the slot taken from block_tables[s]; then out[s] is the
 * attention over context_lens[s] tokens as in pkv_paged_decode_attention.
 * The tensor-core kernel performs the append itself (one launch plus the
 * split-K merge); other shapes run a separate append kernel first.
 */
int pkv_paged_decode_append_attention(void* out, int64_t out_row_stride, const void* q,
                                      int64_t q_row_stride, const void* k_new, const void* v_new,
                                      int64_t k_new_row_stride, int64_t v_new_row_stride,
                                      void* k_pool, void* v_pool, int num_blocks,
                                      const int32_t* block_tables, int64_t block_table_stride,
                                      int max_blocks_per_seq, const int32_t* context_lens,
                                      int n_seqs, int n_q_heads, int n_kv_heads, int head_dim,
                                      int block_size, float scale, int dtype, void* workspace,
                                      size_t workspace_bytes, int* err_flags, pkv_stream_t stream);

/*
 * Paged decode attention for callers that cannot allocate device memory.
 * No counterpart in the reference.  Some hosts of this library cannot call
 * cudaMalloc (or any allocating routine) at the point where they run decode
 * attention -- for example a thin FFI layer that only forwards pointers it
 * was handed, or a process whose device memory is entirely owned by another
 * allocator -- so they cannot provide the split-K workspace that
 * pkv_paged_decode_attention requires.  This entry point takes the same
 * arguments minus the workspace and computes the same result, keeping its
 * split-K partials in a fixed array of PKV_NOALLOC_SCRATCH_BYTES (8 MiB) that
 * is part of the library's device image: every GPU that loads the library
 * holds it until the process exits.  Nothing is allocated per call.
 *  - The first call in each CUDA context looks up that array's device
 *    address (cudaGetSymbolAddress, with that device current) and caches it
 *    under the context's unique id; a context made again after
 *    cudaDeviceReset looks it up again.  Make the first call on a device
 *    (and the first after a reset) before any stream capture.
 *  - Problems whose partials exceed the array (pkv_decode_workspace_bytes >
 *    PKV_NOALLOC_SCRATCH_BYTES, e.g. more than 15 query heads at head_dim 64)
 *    are rejected with PKV_ERR_SCRATCH_LIMIT before anything is launched.
 *  - All calls on a device share the one array and it keeps whatever the
 *    last call left there; nothing in it needs to start at zero (every
 *    partial is written before it is read within a call).  Calls that can
 *    overlap on the GPU (different streams, no ordering) race on it.
 */
int pkv_paged_decode_attention_noalloc(void* out, int64_t out_row_stride, const void* q,
                                       int64_t q_row_stride, const void* k_pool,
                                       const void* v_pool, int num_blocks,
                                       const int32_t* block_tables, int64_t block_table_stride,
                                       int max_blocks_per_seq, const int32_t* context_lens,
                                       int n_seqs, int n_q_heads, int n_kv_heads, int head_dim,
                                       int block_size, float scale, int dtype, int* err_flags,
                                       pkv_stream_t stream);

/*
 * Paged chunked-prefill attention.  Replaces the per-sequence gather +
 * Qwen2Model._attention with num_new > 1 (qwen2.py:98-128): sequence s owns
 * query rows [query_start_loc[s], query_start_loc[s+1]) and its new token i
 * attends to keys 0 .. num_prior[s] + i of the sequence (causal with the
 * reference's num_prior offset; the chunk's own K/V must already be in the
 * pool).  Shared radix-prefix blocks are read in place.  max_query_len bounds
 * query_start_loc[s+1] - query_start_loc[s]; n_tokens >= query_start_loc[n_seqs]:
 * rows from query_start_loc[n_seqs] to n_tokens are padding (a fixed-shape
 * step, e.g. a captured CUDA graph, with fewer real tokens), neither read nor
 * written; a sequence with no rows is skipped.
 */
int pkv_paged_prefill_attention(void* out, int64_t out_row_stride, const void* q,
                                int64_t q_row_stride, const void* k_pool, const void* v_pool,
                                int num_blocks, const int32_t* block_tables,
                                int64_t block_table_stride, int max_blocks_per_seq,
                                const int32_t* query_start_loc, const int32_t* num_prior,
                                int n_seqs, int n_tokens, int max_query_len, int n_q_heads,
                                int n_kv_heads, int head_dim, int block_size, float scale,
                                int dtype, int* err_flags, pkv_stream_t stream);

/*
 * Select the decode kernel for later calls in this process: PKV_DECODE_AUTO
 * (the TMA/tensor-core kernel where the shape allows it) or
 * PKV_DECODE_GENERIC (the portable CUDA-core kernel).  Used by tests that
 * cross-check the two kernels.  No counterpart in the reference.
 */
int pkv_set_decode_impl(int impl);

/*
 * fp8 e4m3 KV pools.  No counterpart in the reference (its quant.py notes fp8
 * KV as the next step after its group-wise absmax int8 weights, with the same
 * math).  Pools hold one byte per element in the reference layout
 * [num_blocks][block_size][n_kv_heads][head_dim]; each (slot, KV head) row has
 * an fp32 scale in k_scale / v_scale [num_blocks * block_size][n_kv_heads]:
 *   scale = absmax(row) / 448 (1 for an all-zero row),
 *   byte  = e4m3(x / scale), round to nearest even, saturated at +-448,
 *   value = e4m3_to_float(byte) * scale.
 * q, out and the arithmetic stay in `dtype`; e4m3 values are exact in fp16.
 */

/* reshape_and_cache into fp8 pools: k, v in `dtype`, quantised per row. */
int pkv_reshape_and_cache_fp8(const void* k, const void* v, int64_t k_row_stride,
                              int64_t v_row_stride, void* k_pool, void* v_pool, float* k_scale,
                              float* v_scale, const int64_t* slot_mapping, int n_tokens,
                              int num_blocks, int block_size, int n_kv_heads, int head_dim,
                              int dtype, int* err_flags, pkv_stream_t stream);

/* pkv_paged_decode_attention over fp8 pools (the new token already
 * appended by pkv_reshape_and_cache_fp8); same workspace contract. */
int pkv_paged_decode_attention_fp8(void* out, int64_t out_row_stride, const void* q,
                                   int64_t q_row_stride, const void* k_pool, const void* v_pool,
                                   const float* k_scale, const float* v_scale, int num_blocks,
                                   const int32_t* block_tables, int64_t block_table_stride,
                                   int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
                                   int n_q_heads, int n_kv_heads, int head_dim, int block_size,
                                   float scale, int dtype, void* workspace, size_t workspace_bytes,
                                   int* err_flags, pkv_stream_t stream);

/* pkv_paged_prefill_attention over fp8 pools (CUDA-core kernel). */
int pkv_paged_prefill_attention_fp8(void* out, int64_t out_row_stride, const void* q,
                                    int64_t q_row_stride, const void* k_pool, const void* v_pool,
                                    const float* k_scale, const float* v_scale, int num_blocks,
                                    const int32_t* block_tables, int64_t block_table_stride,
                                    int max_blocks_per_seq, const int32_t* query_start_loc,
                                    const int32_t* num_prior, int n_seqs, int n_tokens,
                                    int max_query_len, int n_q_heads, int n_kv_heads, int head_dim,
                                    int block_size, float scale, int dtype, int* err_flags,
                                    pkv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGEDKV_H */
