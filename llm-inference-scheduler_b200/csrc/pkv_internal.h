// pkv_internal.h -- host-side launchers shared between the kernel files and
// the C ABI (pkv_abi.cu).  Argument validation happens in pkv_abi.cu; these
// functions assume valid shapes and only launch.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pkv {

// pool format code (internal; not an ABI dtype) of fp8 e4m3 pools, for
// encode_pool_tensormap / pool_tensormap
constexpr int kPoolFp8 = 100;

struct RopeArgs {
  void* q_out;
  int64_t q_out_stride;  // elements between token rows
  const void* qkv;
  int64_t qkv_stride;
  const int64_t* positions;
  const void* cos_t;
  const void* sin_t;
  int max_pos;
  void* k_pool;
  void* v_pool;
  const int64_t* slots;
  int n_tokens, num_blocks, block_size, n_q_heads, n_kv_heads, head_dim, dtype;
  int* err;
  // fp8 e4m3 pools: per-(slot, KV head) scales written with the bytes (NULL: 16/32-bit pools)
  float* k_scale = nullptr;
  float* v_scale = nullptr;
};
cudaError_t launch_rope_reshape_and_cache(const RopeArgs& a, cudaStream_t stream);

struct AttnArgs {
  void* out;
  int64_t out_stride;  // elements between token rows of out
  const void* q;
  int64_t q_stride;    // elements between token rows of q
  const void* k_pool;
  const void* v_pool;
  int num_blocks;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  // decode: context_lens != nullptr, one query row per sequence
  const int32_t* context_lens;
  // prefill: query_start_loc / num_prior
  const int32_t* query_start_loc;
  const int32_t* num_prior;
  int n_seqs;
  int n_tokens;
  int max_query_len;
  int n_q_heads;
  int n_kv_heads;
  int head_dim;
  int block_size;
  float scale;
  int dtype;
  int* err;
  // decode only: the new token of each sequence, written by the decode
  // kernel at position context_lens[s] - 1 before it is read (NULL = none)
  const void* k_new = nullptr;
  const void* v_new = nullptr;
  int64_t k_new_stride = 0;  // elements between rows
  int64_t v_new_stride = 0;
  // fp8 e4m3 pools: one fp32 scale per (slot, KV head); NULL = 16/32-bit pools
  // of `dtype` (q, out and the dequantised arithmetic stay in `dtype`)
  const float* k_scale = nullptr;
  const float* v_scale = nullptr;
  // decode: the step's schedule built by pkv_decode_schedule (NULL = none)
  const void* schedule = nullptr;
  // decode (tensor-core path): a device word the kernel waits on, bounded,
  // until it is nonzero before reading q / k_new / v_new (NULL = none)
  const int* input_ready = nullptr;
  // decode: one layer of a multi-layer call with a workspace per layer (NULL:
  // a single-layer call, its merge launched behind it)
  const struct LayerChain* chain = nullptr;
};

// Layers of one multi-layer decode call, each with its own split-K
// workspace: the decode kernels of layers after the first wait for their
// predecessor only at their end (defer_wait), and one merge launch after the
// last layer's decode covers every layer.
struct LayerChain {
  int defer_wait;            // this layer's decode kernel
  int merge;                 // launch the merge of all n_layers after this decode
  int n_layers;
  void* out0;                // layer 0's output rows
  int64_t out_layer_stride;  // elements between layers' outputs
  void* ws0;                 // layer 0's workspace
  int64_t ws_layer_stride;   // bytes between layers' workspaces
};
cudaError_t launch_reshape_and_cache_fp8(const void* k, const void* v, int64_t k_stride,
                                         int64_t v_stride, void* k_pool, void* v_pool,
                                         float* k_scale, float* v_scale, const int64_t* slots,
                                         int n_tokens, int num_blocks, int block_size,
                                         int n_kv_heads, int head_dim, int src_dtype, int* err,
                                         cudaStream_t stream);

cudaError_t launch_reshape_and_cache(const void* k, const void* v, int64_t k_stride,
                                     int64_t v_stride, void* k_pool, void* v_pool,
                                     const int64_t* slots, int n_tokens, int num_blocks,
                                     int block_size, int n_kv_heads, int head_dim, int esize,
                                     int* err, cudaStream_t stream);

cudaError_t launch_append_at_context_end_fp8(const void* k, const void* v, int64_t k_stride,
                                             int64_t v_stride, void* k_pool, void* v_pool,
                                             float* k_scale, float* v_scale, const int32_t* tables,
                                             int64_t bt_stride, int max_blocks,
                                             const int32_t* context_lens, int n_seqs,
                                             int num_blocks, int block_size, int n_kv_heads,
                                             int head_dim, int src_dtype, int* err,
                                             cudaStream_t stream);
cudaError_t launch_append_at_context_end(const void* k, const void* v, int64_t k_stride,
                                         int64_t v_stride, void* k_pool, void* v_pool,
                                         const int32_t* tables, int64_t bt_stride, int max_blocks,
                                         const int32_t* context_lens, int n_seqs, int num_blocks,
                                         int block_size, int n_kv_heads, int head_dim, int esize,
                                         int* err, cudaStream_t stream);

size_t decode_schedule_bytes(int n_seqs, int max_blocks);
cudaError_t launch_decode_schedule(void* schedule, const AttnArgs& a, cudaStream_t stream);
cudaError_t launch_copy_blocks_peer(void* dst_k, void* dst_v, int64_t dst_layer_stride,
                                    int dst_num_blocks, const void* src_k, const void* src_v,
                                    int64_t src_layer_stride, int src_num_blocks, int n_layers,
                                    const int32_t* pairs, int n_pairs, int64_t block_bytes, int* err,
                                    cudaStream_t stream);
cudaError_t launch_copy_blocks(void* k_pools, void* v_pools, int64_t layer_stride, int n_layers,
                               const int32_t* pairs, int n_pairs, int num_blocks,
                               int64_t block_bytes, int* err, cudaStream_t stream);

// CUDA-core attention for any dtype / head_dim <= 256 / block_size; decode
// (context_lens set) or chunked prefill (query_start_loc + num_prior set).
cudaError_t launch_generic_attention(const AttnArgs& a, cudaStream_t stream);

// Decode fast path: TMA + mbarrier pipeline, tensor-core math, stream-K
// split with fused combine.  Requires fp16/bf16, head_dim 64, block 16,
// n_kv_heads in {1,2,4}, q heads per kv head <= 8.
bool decode_fast_supported(const AttnArgs& a);
bool decode_fast_supported_shape(const AttnArgs& a);
size_t decode_workspace_bytes(int n_seqs, int n_q_heads, int head_dim);
cudaError_t launch_decode_fast(const AttnArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap,
                               void* workspace, cudaStream_t stream);

// TMA descriptor for a pool [num_blocks*block_size][n_kv_heads][head_dim]
// with one (head_dim x 1 head x block_size tokens) box, 128-byte swizzle.
// Returns 0 or a CUresult.
int encode_pool_tensormap(CUtensorMap* map, const void* pool, int num_blocks, int block_size,
                          int n_kv_heads, int head_dim, int dtype);

// Chunked prefill on tcgen05 tensor cores: fp16/bf16, head_dim 64, block 16,
// 16-byte aligned q / out rows.
bool prefill_fast_supported(const AttnArgs& a);
bool prefill_fp8_tc_supported(const AttnArgs& a);
size_t prefill_fp8_scratch_bytes(int n_seqs, int max_blocks, int n_kv_heads, int head_dim);
cudaError_t launch_dequant_blocks(const AttnArgs& a, void* scratch, cudaStream_t stream,
                                  void** k_out, void** v_out, int32_t** table_out);
cudaError_t launch_prefill_fast(const AttnArgs& a, const CUtensorMap* qmap, const CUtensorMap* kmap,
                                const CUtensorMap* vmap, cudaStream_t stream);
// TMA descriptor for q viewed as [n_tokens][n_q_heads][head_dim] (row stride
// q_stride elements) with one (head_dim x 1 head x 128 tokens) box, 128-byte
// swizzle.  Returns 0 or PKV_ERR_DRIVER.
int encode_q_tensormap(CUtensorMap* map, const void* q, int64_t q_stride, int n_tokens,
                       int n_q_heads, int head_dim, int dtype);

// Argument checks, TMA-descriptor cache and kernel selection of pkv_abi.cu,
// reused by the allocation-free decode entry point.
int validate_attention_args(const void* out, int64_t out_stride, const void* q, int64_t q_stride,
                            const void* k_pool, const void* v_pool, int num_blocks,
                            const int32_t* tables, int64_t bt_stride, int max_blocks,
                            int n_q_heads, int n_kv_heads, int head_dim, int block_size, int dtype);
int pool_tensormap(CUtensorMap* out, const void* pool, int num_blocks, int block_size,
                   int n_kv_heads, int head_dim, int dtype);
int decode_impl_setting();

}  // namespace pkv
