// pkv_cache_ops.cu -- KV append (reshape_and_cache) and block copy (copy_blocks).
//
// Both are byte movers bound by HBM bandwidth: rows of n_kv_heads*head_dim
// elements (256 B for the reference's 2 x 64 fp16) move with 16-byte vector
// loads/stores, one warp per token (append) or one CTA per (pair, layer)
// (copy).  Results are bit-exact copies.
#include <algorithm>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

// Append: warp w handles token w.  Lanes cover the K row then the V row in
// 16-byte vectors (row_vecs per row); for 256-byte rows that is exactly one
// vector per lane.  Reference: PagedKVCache.append_and_fetch scatter,
// mini_engine/paged/block_manager.py:121-131.
__global__ void __launch_bounds__(256) reshape_and_cache_vec16(
    const char* __restrict__ k, const char* __restrict__ v, int64_t k_stride_b,
    int64_t v_stride_b, char* __restrict__ k_pool, char* __restrict__ v_pool,
    const int64_t* __restrict__ slots, int n_tokens, int64_t n_slots, int row_bytes, int* err) {
  // launched with programmatic serialization: wait for the preceding grid
  // (its reads of the pool and writes of k / v), then let the next kernel's
  // prologue start
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_tokens) return;
  const int64_t slot = __ldg(slots + warp);
  if (slot < 0) return;  // padding token
  if (slot >= n_slots) {
    if (lane == 0) raise_flag(err, PKV_FLAG_SLOT_OUT_OF_RANGE);
    return;
  }
  const int row_vecs = row_bytes >> 4;
  for (int i = lane; i < 2 * row_vecs; i += 32) {
    const bool is_v = i >= row_vecs;
    const int vi = is_v ? i - row_vecs : i;
    const char* src = (is_v ? v + warp * v_stride_b : k + warp * k_stride_b) + vi * 16;
    char* dst = (is_v ? v_pool : k_pool) + slot * row_bytes + vi * 16;
    const int4 val = __ldg(reinterpret_cast<const int4*>(src));
    __stcs(reinterpret_cast<int4*>(dst), val);
  }
}

// Unaligned fallback: element-sized copies (esize 2 or 4 bytes).
template <typename E>
__global__ void __launch_bounds__(256) reshape_and_cache_elem(
    const E* __restrict__ k, const E* __restrict__ v, int64_t k_stride, int64_t v_stride,
    E* __restrict__ k_pool, E* __restrict__ v_pool, const int64_t* __restrict__ slots,
    int n_tokens, int64_t n_slots, int row_elems, int* err) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n_tokens) return;
  const int64_t slot = slots[warp];
  if (slot < 0) return;
  if (slot >= n_slots) {
    if (lane == 0) raise_flag(err, PKV_FLAG_SLOT_OUT_OF_RANGE);
    return;
  }
  for (int i = lane; i < row_elems; i += 32) {
    k_pool[slot * row_elems + i] = k[warp * k_stride + i];
    v_pool[slot * row_elems + i] = v[warp * v_stride + i];
  }
}

cudaError_t launch_reshape_and_cache(const void* k, const void* v, int64_t k_stride,
                                     int64_t v_stride, void* k_pool, void* v_pool,
                                     const int64_t* slots, int n_tokens, int num_blocks,
                                     int block_size, int n_kv_heads, int head_dim, int esize,
                                     int* err, cudaStream_t stream) {
  if (n_tokens == 0) return cudaSuccess;
  const int row_elems = n_kv_heads * head_dim;
  const int row_bytes = row_elems * esize;
  const int64_t n_slots = static_cast<int64_t>(num_blocks) * block_size;
  const int threads = 256;
  const int grid = (n_tokens + 7) / 8;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = (row_bytes % 16 == 0) && ((k_stride * esize) % 16 == 0) &&
                   ((v_stride * esize) % 16 == 0) && al16(k) && al16(v) && al16(k_pool) &&
                   al16(v_pool);
  if (vec) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, reshape_and_cache_vec16, static_cast<const char*>(k),
                              static_cast<const char*>(v), k_stride * esize, v_stride * esize,
                              static_cast<char*>(k_pool), static_cast<char*>(v_pool), slots,
                              n_tokens, n_slots, row_bytes, err);
  } else if (esize == 4) {
    reshape_and_cache_elem<uint32_t><<<grid, threads, 0, stream>>>(
        static_cast<const uint32_t*>(k), static_cast<const uint32_t*>(v), k_stride, v_stride,
        static_cast<uint32_t*>(k_pool), static_cast<uint32_t*>(v_pool), slots, n_tokens, n_slots,
        row_elems, err);
  } else {
    reshape_and_cache_elem<uint16_t><<<grid, threads, 0, stream>>>(
        static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v), k_stride, v_stride,
        static_cast<uint16_t*>(k_pool), static_cast<uint16_t*>(v_pool), slots, n_tokens, n_slots,
        row_elems, err);
  }
  return cudaGetLastError();
}

// Append one token per sequence at position context_lens[s] - 1, the slot
// taken from the sequence's block table (the decode step's append; used when
// the fused decode kernel does not serve the shape).  One warp per sequence.
template <typename E>
__global__ void __launch_bounds__(256) append_at_context_end(
    const E* __restrict__ k, const E* __restrict__ v, int64_t k_stride, int64_t v_stride,
    E* __restrict__ k_pool, E* __restrict__ v_pool, const int32_t* __restrict__ tables,
    int64_t bt_stride, int max_blocks, const int32_t* __restrict__ context_lens, int n_seqs,
    int num_blocks, int block_size, int row_elems, int* err) {
  const int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (s >= n_seqs) return;
  const int ctx = context_lens[s];
  if (ctx <= 0) return;
  if (ctx > max_blocks * block_size) {
    if (lane == 0) raise_flag(err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
    return;
  }
  const int blk = tables[static_cast<int64_t>(s) * bt_stride + (ctx - 1) / block_size];
  if (blk < 0 || blk >= num_blocks) {
    if (lane == 0) raise_flag(err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
    return;
  }
  const int64_t row = static_cast<int64_t>(blk) * block_size + (ctx - 1) % block_size;
  for (int i = lane; i < row_elems; i += 32) {
    k_pool[row * row_elems + i] = k[s * k_stride + i];
    v_pool[row * row_elems + i] = v[s * v_stride + i];
  }
}

// fp8 e4m3 append: K and V rows quantised per (token, KV head) with scale =
// absmax / 448 (1 for an all-zero row), value = e4m3(x / scale) rounded to
// nearest even and saturated; the byte goes to the pool, the scale to the
// parallel fp32 scale array [slots][n_kv_heads].  One warp per token.
template <typename E>
__global__ void __launch_bounds__(256) reshape_and_cache_fp8_kernel(
    const E* __restrict__ k, const E* __restrict__ v, int64_t k_stride, int64_t v_stride,
    uint8_t* __restrict__ k_pool, uint8_t* __restrict__ v_pool, float* __restrict__ k_scale,
    float* __restrict__ v_scale, const int64_t* __restrict__ slots, int n_tokens, int64_t n_slots,
    int hkv, int d, int* err) {
  pdl_wait();
  pdl_trigger();
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= n_tokens) return;
  const int64_t slot = __ldg(slots + t);
  if (slot < 0) return;  // padding token
  if (slot >= n_slots) {
    if (lane == 0) raise_flag(err, PKV_FLAG_SLOT_OUT_OF_RANGE);
    return;
  }
  fp8_store_token<E>(k + t * k_stride, k_pool + slot * hkv * d, k_scale + slot * hkv, hkv, d, lane);
  fp8_store_token<E>(v + t * v_stride, v_pool + slot * hkv * d, v_scale + slot * hkv, hkv, d, lane);
}

// append_at_context_end into fp8 pools: the quantising append of
// reshape_and_cache_fp8 at the slot of each sequence's newest token.
template <typename E>
__global__ void __launch_bounds__(256) append_at_context_end_fp8(
    const E* __restrict__ k, const E* __restrict__ v, int64_t k_stride, int64_t v_stride,
    uint8_t* __restrict__ k_pool, uint8_t* __restrict__ v_pool, float* __restrict__ k_scale,
    float* __restrict__ v_scale, const int32_t* __restrict__ tables, int64_t bt_stride,
    int max_blocks, const int32_t* __restrict__ context_lens, int n_seqs, int num_blocks,
    int block_size, int hkv, int d, int* err) {
  const int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (s >= n_seqs) return;
  const int ctx = context_lens[s];
  if (ctx <= 0) return;
  if (ctx > max_blocks * block_size) {
    if (lane == 0) raise_flag(err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
    return;
  }
  const int blk = tables[static_cast<int64_t>(s) * bt_stride + (ctx - 1) / block_size];
  if (blk < 0 || blk >= num_blocks) {
    if (lane == 0) raise_flag(err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
    return;
  }
  const int64_t slot = static_cast<int64_t>(blk) * block_size + (ctx - 1) % block_size;
  fp8_store_token<E>(k + s * k_stride, k_pool + slot * hkv * d, k_scale + slot * hkv, hkv, d, lane);
  fp8_store_token<E>(v + s * v_stride, v_pool + slot * hkv * d, v_scale + slot * hkv, hkv, d, lane);
}

cudaError_t launch_append_at_context_end_fp8(const void* k, const void* v, int64_t k_stride,
                                             int64_t v_stride, void* k_pool, void* v_pool,
                                             float* k_scale, float* v_scale, const int32_t* tables,
                                             int64_t bt_stride, int max_blocks,
                                             const int32_t* context_lens, int n_seqs,
                                             int num_blocks, int block_size, int n_kv_heads,
                                             int head_dim, int src_dtype, int* err,
                                             cudaStream_t stream) {
  if (n_seqs == 0) return cudaSuccess;
  const int grid = (n_seqs + 7) / 8;
  auto go = [&](auto tag) {
    using E = decltype(tag);
    append_at_context_end_fp8<E><<<grid, 256, 0, stream>>>(
        static_cast<const E*>(k), static_cast<const E*>(v), k_stride, v_stride,
        static_cast<uint8_t*>(k_pool), static_cast<uint8_t*>(v_pool), k_scale, v_scale, tables,
        bt_stride, max_blocks, context_lens, n_seqs, num_blocks, block_size, n_kv_heads, head_dim,
        err);
    return cudaGetLastError();
  };
  if (src_dtype == PKV_DTYPE_F32) return go(float{});
  if (src_dtype == PKV_DTYPE_F16) return go(__half{});
  return go(__nv_bfloat16{});
}

cudaError_t launch_reshape_and_cache_fp8(const void* k, const void* v, int64_t k_stride,
                                         int64_t v_stride, void* k_pool, void* v_pool,
                                         float* k_scale, float* v_scale, const int64_t* slots,
                                         int n_tokens, int num_blocks, int block_size,
                                         int n_kv_heads, int head_dim, int src_dtype, int* err,
                                         cudaStream_t stream) {
  if (n_tokens == 0) return cudaSuccess;
  const int64_t n_slots = static_cast<int64_t>(num_blocks) * block_size;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((n_tokens + 7) / 8);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto go = [&](auto tag) {
    using E = decltype(tag);
    return cudaLaunchKernelEx(&cfg, reshape_and_cache_fp8_kernel<E>, static_cast<const E*>(k),
                              static_cast<const E*>(v), k_stride, v_stride,
                              static_cast<uint8_t*>(k_pool), static_cast<uint8_t*>(v_pool), k_scale,
                              v_scale, slots, n_tokens, n_slots, n_kv_heads, head_dim, err);
  };
  if (src_dtype == PKV_DTYPE_F32) return go(float{});
  if (src_dtype == PKV_DTYPE_F16) return go(__half{});
  return go(__nv_bfloat16{});
}

cudaError_t launch_append_at_context_end(const void* k, const void* v, int64_t k_stride,
                                         int64_t v_stride, void* k_pool, void* v_pool,
                                         const int32_t* tables, int64_t bt_stride, int max_blocks,
                                         const int32_t* context_lens, int n_seqs, int num_blocks,
                                         int block_size, int n_kv_heads, int head_dim, int esize,
                                         int* err, cudaStream_t stream) {
  if (n_seqs == 0) return cudaSuccess;
  const int grid = (n_seqs + 7) / 8;
  const int row = n_kv_heads * head_dim;
  if (esize == 4)
    append_at_context_end<uint32_t><<<grid, 256, 0, stream>>>(
        static_cast<const uint32_t*>(k), static_cast<const uint32_t*>(v), k_stride, v_stride,
        static_cast<uint32_t*>(k_pool), static_cast<uint32_t*>(v_pool), tables, bt_stride,
        max_blocks, context_lens, n_seqs, num_blocks, block_size, row, err);
  else
    append_at_context_end<uint16_t><<<grid, 256, 0, stream>>>(
        static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v), k_stride, v_stride,
        static_cast<uint16_t*>(k_pool), static_cast<uint16_t*>(v_pool), tables, bt_stride,
        max_blocks, context_lens, n_seqs, num_blocks, block_size, row, err);
  return cudaGetLastError();
}

// Copy: CTA (pair p, layer l) copies K block then V block of that layer.
// Reference: BlockManager.copy_block, mini_engine/paged/block_manager.py:65-71.
__global__ void __launch_bounds__(256) copy_blocks_vec16(char* __restrict__ k_pools,
                                                         char* __restrict__ v_pools,
                                                         int64_t layer_stride,
                                                         const int32_t* __restrict__ pairs,
                                                         int num_blocks, int64_t block_bytes,
                                                         int* err) {
  const int p = blockIdx.x;
  const int layer = blockIdx.y;
  const int src = __ldg(pairs + 2 * p), dst = __ldg(pairs + 2 * p + 1);
  if (src < 0 || dst < 0 || src >= num_blocks || dst >= num_blocks) {
    if (threadIdx.x == 0 && layer == 0) raise_flag(err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
    return;
  }
  const int64_t nvec = block_bytes >> 4;
  const int64_t base = layer * layer_stride;
  const int4* ks = reinterpret_cast<const int4*>(k_pools + base + src * block_bytes);
  const int4* vs = reinterpret_cast<const int4*>(v_pools + base + src * block_bytes);
  int4* kd = reinterpret_cast<int4*>(k_pools + base + dst * block_bytes);
  int4* vd = reinterpret_cast<int4*>(v_pools + base + dst * block_bytes);
  for (int64_t i = threadIdx.x; i < nvec; i += blockDim.x) {
    const int4 a = ks[i];
    const int4 b = vs[i];
    kd[i] = a;
    vd[i] = b;
  }
}

__global__ void __launch_bounds__(256) copy_blocks_bytes(char* __restrict__ k_pools,
                                                         char* __restrict__ v_pools,
                                                         int64_t layer_stride,
                                                         const int32_t* __restrict__ pairs,
                                                         int num_blocks, int64_t block_bytes,
                                                         int* err) {
  const int p = blockIdx.x;
  const int layer = blockIdx.y;
  const int src = pairs[2 * p], dst = pairs[2 * p + 1];
  if (src < 0 || dst < 0 || src >= num_blocks || dst >= num_blocks) {
    if (threadIdx.x == 0 && layer == 0) raise_flag(err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
    return;
  }
  const int64_t base = layer * layer_stride;
  for (int64_t i = threadIdx.x; i < block_bytes; i += blockDim.x) {
    k_pools[base + dst * block_bytes + i] = k_pools[base + src * block_bytes + i];
    v_pools[base + dst * block_bytes + i] = v_pools[base + src * block_bytes + i];
  }
}

// Block copy between two pools that may live on different GPUs: one of them
// (or both) mapped from a peer process with CUDA IPC, so the loads or the
// stores cross NVLink.  Used for KV block migration between ranks (a rank
// pulls a peer's blocks, or pushes its own into a peer's pool) in place of
// recompute preemption (mini_engine/scheduler.py:143-156 drops the KV and
// recomputes it).  Plain 16-byte loads and stores only, no TMA.
// One CTA per (pair, layer); each thread issues all its loads before its
// stores, so a CTA keeps the whole K and V block in flight over the link.
constexpr int kPeerVecsPerThread = 4;
__global__ void __launch_bounds__(256) copy_blocks_peer_vec16(
    char* __restrict__ dst_k, char* __restrict__ dst_v, int64_t dst_layer_stride, int dst_num_blocks,
    const char* __restrict__ src_k, const char* __restrict__ src_v, int64_t src_layer_stride,
    int src_num_blocks, const int32_t* __restrict__ pairs, int64_t block_bytes, int* err) {
  const int p = blockIdx.x;
  const int layer = blockIdx.y;
  const int src = __ldg(pairs + 2 * p), dst = __ldg(pairs + 2 * p + 1);
  if (src < 0 || dst < 0 || src >= src_num_blocks || dst >= dst_num_blocks) {
    if (threadIdx.x == 0 && layer == 0) raise_flag(err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
    return;
  }
  const int64_t nvec = block_bytes >> 4;
  const int4* ks = reinterpret_cast<const int4*>(src_k + layer * src_layer_stride + src * block_bytes);
  const int4* vs = reinterpret_cast<const int4*>(src_v + layer * src_layer_stride + src * block_bytes);
  int4* kd = reinterpret_cast<int4*>(dst_k + layer * dst_layer_stride + dst * block_bytes);
  int4* vd = reinterpret_cast<int4*>(dst_v + layer * dst_layer_stride + dst * block_bytes);
  for (int64_t i0 = threadIdx.x; i0 < nvec; i0 += static_cast<int64_t>(blockDim.x) * kPeerVecsPerThread) {
    int4 a[kPeerVecsPerThread], b[kPeerVecsPerThread];
#pragma unroll
    for (int j = 0; j < kPeerVecsPerThread; ++j) {
      const int64_t i = i0 + static_cast<int64_t>(j) * blockDim.x;
      if (i < nvec) {
        a[j] = ks[i];
        b[j] = vs[i];
      }
    }
#pragma unroll
    for (int j = 0; j < kPeerVecsPerThread; ++j) {
      const int64_t i = i0 + static_cast<int64_t>(j) * blockDim.x;
      if (i < nvec) {
        kd[i] = a[j];
        vd[i] = b[j];
      }
    }
  }
}

cudaError_t launch_copy_blocks_peer(void* dst_k, void* dst_v, int64_t dst_layer_stride,
                                    int dst_num_blocks, const void* src_k, const void* src_v,
                                    int64_t src_layer_stride, int src_num_blocks, int n_layers,
                                    const int32_t* pairs, int n_pairs, int64_t block_bytes, int* err,
                                    cudaStream_t stream) {
  if (n_pairs == 0 || n_layers == 0) return cudaSuccess;
  const int64_t nvec = block_bytes >> 4;
  // enough threads for the block's vectors, a multiple of a warp, at most 256
  const int threads = static_cast<int>(std::min<int64_t>(256, std::max<int64_t>(32, (nvec + 31) / 32 * 32)));
  copy_blocks_peer_vec16<<<dim3(n_pairs, n_layers), threads, 0, stream>>>(
      static_cast<char*>(dst_k), static_cast<char*>(dst_v), dst_layer_stride, dst_num_blocks,
      static_cast<const char*>(src_k), static_cast<const char*>(src_v), src_layer_stride,
      src_num_blocks, pairs, block_bytes, err);
  return cudaGetLastError();
}

cudaError_t launch_copy_blocks(void* k_pools, void* v_pools, int64_t layer_stride, int n_layers,
                               const int32_t* pairs, int n_pairs, int num_blocks,
                               int64_t block_bytes, int* err, cudaStream_t stream) {
  if (n_pairs == 0 || n_layers == 0) return cudaSuccess;
  dim3 grid(n_pairs, n_layers);
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (block_bytes % 16 == 0 && layer_stride % 16 == 0 && al16(k_pools) && al16(v_pools)) {
    copy_blocks_vec16<<<grid, 256, 0, stream>>>(static_cast<char*>(k_pools),
                                                static_cast<char*>(v_pools), layer_stride, pairs,
                                                num_blocks, block_bytes, err);
  } else {
    copy_blocks_bytes<<<grid, 256, 0, stream>>>(static_cast<char*>(k_pools),
                                                static_cast<char*>(v_pools), layer_stride, pairs,
                                                num_blocks, block_bytes, err);
  }
  return cudaGetLastError();
}

}  // namespace pkv
