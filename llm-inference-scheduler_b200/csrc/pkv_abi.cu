// pkv_abi.cu -- the extern "C" entry points of libpagedkv.so (include/pagedkv.h).
//
// Each entry point validates its arguments on the host (returning a negative
// PKV_ERR_* code before anything is launched), picks a kernel, and launches
// it on the caller's stream.  Nothing here allocates device memory or
// synchronises.  TMA descriptors for pool tensors are encoded through the
// driver entry point cuTensorMapEncodeTiled and cached per pool pointer.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;
std::once_flag g_addr_range_once;

PFN_cuMemGetAddressRange_v3020 address_range() {
  std::call_once(g_addr_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &fn, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  return g_addr_range;
}

static_assert(sizeof(cudaIpcMemHandle_t) == PKV_IPC_HANDLE_BYTES, "CUDA IPC handle size");

struct MapKey {
  const void* ptr;
  int num_blocks, block_size, n_kv_heads, head_dim, dtype;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && num_blocks == o.num_blocks && block_size == o.block_size &&
           n_kv_heads == o.n_kv_heads && head_dim == o.head_dim && dtype == o.dtype;
  }
};
struct MapHash {
  size_t operator()(const MapKey& k) const {
    size_t h = reinterpret_cast<size_t>(k.ptr);
    h ^= (static_cast<size_t>(k.num_blocks) << 20) ^ (static_cast<size_t>(k.dtype) << 60) ^
         (static_cast<size_t>(k.n_kv_heads) << 52) ^ (static_cast<size_t>(k.head_dim) << 44);
    return h * 0x9E3779B97F4A7C15ull;
  }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapHash> g_maps;
constexpr size_t kMaxCachedMaps = 4096;

int cached_pool_map(CUtensorMap* out, const void* pool, int num_blocks, int block_size,
                    int n_kv_heads, int head_dim, int dtype) {
  const MapKey key{pool, num_blocks, block_size, n_kv_heads, head_dim, dtype};
  std::lock_guard<std::mutex> lk(g_map_mu);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return 0;
  }
  CUtensorMap m;
  const int rc = encode_pool_tensormap(&m, pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
  if (rc != 0) return rc;
  if (g_maps.size() >= kMaxCachedMaps) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return 0;
}

std::atomic<int> g_decode_impl{PKV_DECODE_AUTO};

inline bool valid_dtype(int dt) { return dt == PKV_DTYPE_F32 || dt == PKV_DTYPE_F16 || dt == PKV_DTYPE_BF16; }
inline int esize_of(int dt) { return dt == PKV_DTYPE_F32 ? 4 : 2; }

int status_of(cudaError_t e) { return e == cudaSuccess ? PKV_OK : static_cast<int>(e); }

// shared shape checks of the two attention entry points
int check_attn(const void* out, int64_t out_stride, const void* q, int64_t q_stride,
               const void* k_pool, const void* v_pool, int num_blocks, const int32_t* tables,
               int64_t bt_stride, int max_blocks, int n_q_heads, int n_kv_heads, int head_dim,
               int block_size, int dtype) {
  if (!out || !q || !k_pool || !v_pool || !tables) return PKV_ERR_NULL_POINTER;
  if (!valid_dtype(dtype)) return PKV_ERR_BAD_DTYPE;
  if (n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0) return PKV_ERR_BAD_SHAPE;
  if (head_dim <= 0 || head_dim > 256 || block_size <= 0 || num_blocks <= 0 || max_blocks <= 0)
    return PKV_ERR_BAD_SHAPE;
  if (bt_stride < max_blocks) return PKV_ERR_BAD_SHAPE;
  const int64_t row = static_cast<int64_t>(n_q_heads) * head_dim;
  if (q_stride < row || out_stride < row) return PKV_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(max_blocks) * block_size > 0x7fffffff) return PKV_ERR_BAD_SHAPE;
  if (static_cast<int64_t>(num_blocks) * block_size > 0x7fffffff) return PKV_ERR_BAD_SHAPE;
  return PKV_OK;
}

// tensor-core decode when the shape allows it (16-bit or fp8 pools), else the
// CUDA-core kernel
int decode_dispatch(AttnArgs& a, void* workspace, size_t workspace_bytes, cudaStream_t st) {
  if (g_decode_impl.load() == PKV_DECODE_AUTO && decode_fast_supported(a)) {
    if (!workspace) return PKV_ERR_NULL_POINTER;
    if (workspace_bytes < decode_workspace_bytes(a.n_seqs, a.n_q_heads, a.head_dim))
      return PKV_ERR_WORKSPACE_TOO_SMALL;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return PKV_ERR_MISALIGNED;
    const int fmt = a.k_scale != nullptr ? kPoolFp8 : a.dtype;
    CUtensorMap km, vm;
    int rc = cached_pool_map(&km, a.k_pool, a.num_blocks, a.block_size, a.n_kv_heads, a.head_dim, fmt);
    if (rc != 0) return rc;
    rc = cached_pool_map(&vm, a.v_pool, a.num_blocks, a.block_size, a.n_kv_heads, a.head_dim, fmt);
    if (rc != 0) return rc;
    return status_of(launch_decode_fast(a, &km, &vm, workspace, st));
  }
  return status_of(launch_generic_attention(a, st));
}

}  // namespace

// Shared with the allocation-free decode entry point (pkv_decode_noalloc.cu).
int validate_attention_args(const void* out, int64_t out_stride, const void* q, int64_t q_stride,
                            const void* k_pool, const void* v_pool, int num_blocks,
                            const int32_t* tables, int64_t bt_stride, int max_blocks,
                            int n_q_heads, int n_kv_heads, int head_dim, int block_size, int dtype) {
  return check_attn(out, out_stride, q, q_stride, k_pool, v_pool, num_blocks, tables, bt_stride,
                    max_blocks, n_q_heads, n_kv_heads, head_dim, block_size, dtype);
}
int pool_tensormap(CUtensorMap* out, const void* pool, int num_blocks, int block_size,
                   int n_kv_heads, int head_dim, int dtype) {
  return cached_pool_map(out, pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
}
int decode_impl_setting() { return g_decode_impl.load(); }

int encode_pool_tensormap(CUtensorMap* map, const void* pool, int num_blocks, int block_size,
                          int n_kv_heads, int head_dim, int dtype) {
  auto enc = encoder();
  if (enc == nullptr) return PKV_ERR_DRIVER;
  // 16-bit pools: 128-byte rows with the 128-byte swizzle (ldmatrix reads them
  // in place); fp8 pools: 64-byte rows, unswizzled (converted by the consumers)
  const bool fp8 = dtype == kPoolFp8;
  const cuuint64_t es = fp8 ? 1 : 2;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(n_kv_heads),
                              static_cast<cuuint64_t>(num_blocks) * block_size};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim) * es,
                                 static_cast<cuuint64_t>(n_kv_heads) * head_dim * es};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(head_dim), 1u, static_cast<cuuint32_t>(block_size)};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt = fp8                      ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : dtype == PKV_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUresult r = enc(map, dt, 3, const_cast<void*>(pool), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         fp8 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : PKV_ERR_DRIVER;
}

int encode_q_tensormap(CUtensorMap* map, const void* q, int64_t q_stride, int n_tokens,
                       int n_q_heads, int head_dim, int dtype) {
  auto enc = encoder();
  if (enc == nullptr) return PKV_ERR_DRIVER;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(n_q_heads),
                              static_cast<cuuint64_t>(n_tokens)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim) * 2,
                                 static_cast<cuuint64_t>(q_stride) * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(head_dim), 1u, 128u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUtensorMapDataType dt =
      dtype == PKV_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUresult r = enc(map, dt, 3, const_cast<void*>(q), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : PKV_ERR_DRIVER;
}

}  // namespace pkv

using namespace pkv;

extern "C" {

int pkv_abi_version(void) { return PKV_ABI_VERSION; }

const char* pkv_status_string(int status) {
  switch (status) {
    case PKV_OK: return "ok";
    case PKV_ERR_NULL_POINTER: return "a required pointer argument is NULL";
    case PKV_ERR_BAD_SHAPE: return "inconsistent or out-of-range shape argument";
    case PKV_ERR_BAD_DTYPE: return "dtype must be PKV_DTYPE_F32, PKV_DTYPE_F16 or PKV_DTYPE_BF16";
    case PKV_ERR_WORKSPACE_TOO_SMALL: return "workspace smaller than pkv_decode_workspace_bytes()";
    case PKV_ERR_MISALIGNED: return "pointer or stride misaligned for this kernel";
    case PKV_ERR_UNSUPPORTED: return "combination of arguments not supported";
    case PKV_ERR_DRIVER:
      return "a CUDA driver entry point (cuTensorMapEncodeTiled, cuMemGetAddressRange, "
             "cuCtxGetCurrent, cuCtxGetId) is unavailable or failed";
    case PKV_ERR_SCRATCH_LIMIT:
      return "problem needs more split-K scratch than the allocation-free decode entry point's "
             "fixed PKV_NOALLOC_SCRATCH_BYTES array holds; use pkv_paged_decode_attention";
    default: break;
  }
  if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
  return "unknown pagedkv status";
}

int pkv_set_decode_impl(int impl) {
  if (impl != PKV_DECODE_AUTO && impl != PKV_DECODE_GENERIC) return PKV_ERR_UNSUPPORTED;
  g_decode_impl.store(impl);
  return PKV_OK;
}

int pkv_reshape_and_cache(const void* k, const void* v, int64_t k_row_stride, int64_t v_row_stride,
                          void* k_pool, void* v_pool, const int64_t* slot_mapping, int n_tokens,
                          int num_blocks, int block_size, int n_kv_heads, int head_dim, int dtype,
                          int* err_flags, pkv_stream_t stream) {
  if (n_tokens < 0) return PKV_ERR_BAD_SHAPE;
  if (n_tokens == 0) return PKV_OK;
  if (!k || !v || !k_pool || !v_pool || !slot_mapping) return PKV_ERR_NULL_POINTER;
  if (!valid_dtype(dtype)) return PKV_ERR_BAD_DTYPE;
  if (num_blocks <= 0 || block_size <= 0 || n_kv_heads <= 0 || head_dim <= 0) return PKV_ERR_BAD_SHAPE;
  const int64_t row = static_cast<int64_t>(n_kv_heads) * head_dim;
  if (k_row_stride < row || v_row_stride < row) return PKV_ERR_BAD_SHAPE;
  return status_of(launch_reshape_and_cache(k, v, k_row_stride, v_row_stride, k_pool, v_pool,
                                            slot_mapping, n_tokens, num_blocks, block_size,
                                            n_kv_heads, head_dim, esize_of(dtype), err_flags,
                                            static_cast<cudaStream_t>(stream)));
}

int pkv_reshape_and_cache_fp8(const void* k, const void* v, int64_t k_row_stride,
                              int64_t v_row_stride, void* k_pool, void* v_pool, float* k_scale,
                              float* v_scale, const int64_t* slot_mapping, int n_tokens,
                              int num_blocks, int block_size, int n_kv_heads, int head_dim,
                              int dtype, int* err_flags, pkv_stream_t stream) {
  if (n_tokens < 0) return PKV_ERR_BAD_SHAPE;
  if (n_tokens == 0) return PKV_OK;
  if (!k || !v || !k_pool || !v_pool || !k_scale || !v_scale || !slot_mapping)
    return PKV_ERR_NULL_POINTER;
  if (!valid_dtype(dtype)) return PKV_ERR_BAD_DTYPE;
  if (num_blocks <= 0 || block_size <= 0 || n_kv_heads <= 0 || head_dim <= 0) return PKV_ERR_BAD_SHAPE;
  const int64_t row = static_cast<int64_t>(n_kv_heads) * head_dim;
  if (k_row_stride < row || v_row_stride < row) return PKV_ERR_BAD_SHAPE;
  return status_of(launch_reshape_and_cache_fp8(k, v, k_row_stride, v_row_stride, k_pool, v_pool,
                                                k_scale, v_scale, slot_mapping, n_tokens, num_blocks,
                                                block_size, n_kv_heads, head_dim, dtype, err_flags,
                                                static_cast<cudaStream_t>(stream)));
}

static int rope_entry(void* q_out, int64_t q_out_row_stride, const void* qkv,
                      int64_t qkv_row_stride, const int64_t* positions, const void* cos_table,
                      const void* sin_table, int max_position, void* k_pool, void* v_pool,
                      float* k_scale, float* v_scale, const int64_t* slot_mapping, int n_tokens,
                      int num_blocks, int block_size, int n_q_heads, int n_kv_heads, int head_dim,
                      int dtype, int* err_flags, pkv_stream_t stream) {
  if (n_tokens < 0) return PKV_ERR_BAD_SHAPE;
  if (n_tokens == 0) return PKV_OK;
  if (!q_out || !qkv || !positions || !cos_table || !sin_table || !k_pool || !v_pool ||
      !slot_mapping)
    return PKV_ERR_NULL_POINTER;
  if (!valid_dtype(dtype)) return PKV_ERR_BAD_DTYPE;
  if (num_blocks <= 0 || block_size <= 0 || n_q_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 ||
      (head_dim & 1) || max_position <= 0)
    return PKV_ERR_BAD_SHAPE;
  if (q_out_row_stride < static_cast<int64_t>(n_q_heads) * head_dim ||
      qkv_row_stride < static_cast<int64_t>(n_q_heads + 2 * n_kv_heads) * head_dim)
    return PKV_ERR_BAD_SHAPE;
  RopeArgs a{};
  a.q_out = q_out;
  a.q_out_stride = q_out_row_stride;
  a.qkv = qkv;
  a.qkv_stride = qkv_row_stride;
  a.positions = positions;
  a.cos_t = cos_table;
  a.sin_t = sin_table;
  a.max_pos = max_position;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.slots = slot_mapping;
  a.n_tokens = n_tokens;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.dtype = dtype;
  a.err = err_flags;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  return status_of(launch_rope_reshape_and_cache(a, static_cast<cudaStream_t>(stream)));
}

int pkv_rope_reshape_and_cache(void* q_out, int64_t q_out_row_stride, const void* qkv,
                               int64_t qkv_row_stride, const int64_t* positions,
                               const void* cos_table, const void* sin_table, int max_position,
                               void* k_pool, void* v_pool, const int64_t* slot_mapping,
                               int n_tokens, int num_blocks, int block_size, int n_q_heads,
                               int n_kv_heads, int head_dim, int dtype, int* err_flags,
                               pkv_stream_t stream) {
  return rope_entry(q_out, q_out_row_stride, qkv, qkv_row_stride, positions, cos_table, sin_table,
                    max_position, k_pool, v_pool, nullptr, nullptr, slot_mapping, n_tokens,
                    num_blocks, block_size, n_q_heads, n_kv_heads, head_dim, dtype, err_flags,
                    stream);
}

int pkv_rope_reshape_and_cache_fp8(void* q_out, int64_t q_out_row_stride, const void* qkv,
                                   int64_t qkv_row_stride, const int64_t* positions,
                                   const void* cos_table, const void* sin_table, int max_position,
                                   void* k_pool, void* v_pool, float* k_scale, float* v_scale,
                                   const int64_t* slot_mapping, int n_tokens, int num_blocks,
                                   int block_size, int n_q_heads, int n_kv_heads, int head_dim,
                                   int dtype, int* err_flags, pkv_stream_t stream) {
  if (n_tokens > 0 && (!k_scale || !v_scale)) return PKV_ERR_NULL_POINTER;
  return rope_entry(q_out, q_out_row_stride, qkv, qkv_row_stride, positions, cos_table, sin_table,
                    max_position, k_pool, v_pool, k_scale, v_scale, slot_mapping, n_tokens,
                    num_blocks, block_size, n_q_heads, n_kv_heads, head_dim, dtype, err_flags,
                    stream);
}

int pkv_copy_blocks(void* k_pools, void* v_pools, int64_t layer_stride_bytes, int n_layers,
                    const int32_t* block_pairs, int n_pairs, int num_blocks, int64_t block_bytes,
                    int* err_flags, pkv_stream_t stream) {
  if (n_pairs < 0 || n_layers < 0) return PKV_ERR_BAD_SHAPE;
  if (n_pairs == 0 || n_layers == 0) return PKV_OK;
  if (!k_pools || !v_pools || !block_pairs) return PKV_ERR_NULL_POINTER;
  if (num_blocks <= 0 || block_bytes <= 0) return PKV_ERR_BAD_SHAPE;
  if (n_layers > 65535) return PKV_ERR_UNSUPPORTED;
  if (n_layers > 1 && layer_stride_bytes < static_cast<int64_t>(num_blocks) * block_bytes)
    return PKV_ERR_BAD_SHAPE;
  return status_of(launch_copy_blocks(k_pools, v_pools, layer_stride_bytes, n_layers, block_pairs,
                                      n_pairs, num_blocks, block_bytes, err_flags,
                                      static_cast<cudaStream_t>(stream)));
}

int pkv_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset) {
  if (!dev_ptr || !handle || !offset) return PKV_ERR_NULL_POINTER;
  auto range = address_range();
  if (range == nullptr) return PKV_ERR_DRIVER;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return PKV_ERR_DRIVER;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return status_of(e);
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(dev_ptr) - base);
  return PKV_OK;
}

int pkv_ipc_open(const void* handle, void** base) {
  if (!handle || !base) return PKV_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return status_of(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
}

int pkv_ipc_close(void* base) {
  if (!base) return PKV_ERR_NULL_POINTER;
  return status_of(cudaIpcCloseMemHandle(base));
}

int pkv_copy_blocks_peer(void* dst_k, void* dst_v, int64_t dst_layer_stride_bytes,
                         int dst_num_blocks, const void* src_k, const void* src_v,
                         int64_t src_layer_stride_bytes, int src_num_blocks, int n_layers,
                         const int32_t* block_pairs, int n_pairs, int64_t block_bytes,
                         int* err_flags, pkv_stream_t stream) {
  if (n_pairs < 0 || n_layers < 0) return PKV_ERR_BAD_SHAPE;
  if (n_pairs == 0 || n_layers == 0) return PKV_OK;
  if (!dst_k || !dst_v || !src_k || !src_v || !block_pairs) return PKV_ERR_NULL_POINTER;
  if (dst_num_blocks <= 0 || src_num_blocks <= 0 || block_bytes <= 0) return PKV_ERR_BAD_SHAPE;
  if (n_layers > 65535) return PKV_ERR_UNSUPPORTED;
  if (n_layers > 1 && (dst_layer_stride_bytes < static_cast<int64_t>(dst_num_blocks) * block_bytes ||
                       src_layer_stride_bytes < static_cast<int64_t>(src_num_blocks) * block_bytes))
    return PKV_ERR_BAD_SHAPE;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (block_bytes % 16 || dst_layer_stride_bytes % 16 || src_layer_stride_bytes % 16 || !al16(dst_k) ||
      !al16(dst_v) || !al16(src_k) || !al16(src_v))
    return PKV_ERR_MISALIGNED;
  return status_of(launch_copy_blocks_peer(dst_k, dst_v, dst_layer_stride_bytes, dst_num_blocks, src_k,
                                           src_v, src_layer_stride_bytes, src_num_blocks, n_layers,
                                           block_pairs, n_pairs, block_bytes, err_flags,
                                           static_cast<cudaStream_t>(stream)));
}

size_t pkv_decode_schedule_bytes(int n_seqs, int max_blocks_per_seq) {
  if (n_seqs < 0 || max_blocks_per_seq < 0) return 0;
  return decode_schedule_bytes(n_seqs, max_blocks_per_seq);
}

int pkv_decode_schedule(void* schedule, size_t schedule_bytes, const int32_t* block_tables,
                        int64_t block_table_stride, int max_blocks_per_seq,
                        const int32_t* context_lens, int n_seqs, int num_blocks, int n_q_heads,
                        int n_kv_heads, int head_dim, int block_size, int dtype, int fp8_pools,
                        int* err_flags, pkv_stream_t stream) {
  if (n_seqs < 0 || max_blocks_per_seq < 0) return PKV_ERR_BAD_SHAPE;
  if (!schedule || !block_tables || !context_lens) return PKV_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(schedule) & 15) != 0) return PKV_ERR_MISALIGNED;
  if (schedule_bytes < decode_schedule_bytes(n_seqs, max_blocks_per_seq))
    return PKV_ERR_WORKSPACE_TOO_SMALL;
  if (n_seqs > 2048 || n_kv_heads <= 0 || n_q_heads % n_kv_heads != 0 || num_blocks <= 0 ||
      block_table_stride < max_blocks_per_seq)
    return PKV_ERR_BAD_SHAPE;
  if (dtype != PKV_DTYPE_F32 && dtype != PKV_DTYPE_F16 && dtype != PKV_DTYPE_BF16)
    return PKV_ERR_BAD_DTYPE;
  if (n_seqs == 0) return PKV_OK;
  AttnArgs a{};
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  a.n_seqs = n_seqs;
  a.num_blocks = num_blocks;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.dtype = dtype;
  a.err = err_flags;
  static const float kOne = 1.f;  // marks fp8 pools for the grid choice only
  if (fp8_pools) a.k_scale = a.v_scale = &kOne;
  // the schedule serves the tensor-core kernel only; other shapes ignore it
  if (!(decode_fast_supported_shape(a))) return PKV_OK;
  return status_of(launch_decode_schedule(schedule, a, static_cast<cudaStream_t>(stream)));
}

size_t pkv_decode_workspace_bytes(int n_seqs, int n_q_heads, int head_dim) {
  if (n_seqs < 0 || n_q_heads <= 0 || head_dim <= 0) return 0;
  return decode_workspace_bytes(n_seqs, n_q_heads, head_dim);
}

static int pkv_paged_decode_attention_impl(void* out, int64_t out_row_stride, const void* q,
                                           int64_t q_row_stride, const void* k_pool,
                                           const void* v_pool, int num_blocks,
                                           const int32_t* block_tables, int64_t block_table_stride,
                                           int max_blocks_per_seq, const int32_t* context_lens,
                                           int n_seqs, int n_q_heads, int n_kv_heads, int head_dim,
                                           int block_size, float scale, int dtype, void* workspace,
                                           size_t workspace_bytes, int* err_flags,
                                           pkv_stream_t stream, const void* schedule) {
  if (n_seqs < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!context_lens) return PKV_ERR_NULL_POINTER;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  a.n_seqs = n_seqs;
  a.n_tokens = n_seqs;
  a.max_query_len = 1;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  a.schedule = schedule;
  return decode_dispatch(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

static int pkv_paged_decode_attention_fp8_impl(void* out, int64_t out_row_stride, const void* q,
                                               int64_t q_row_stride, const void* k_pool,
                                               const void* v_pool, const float* k_scale,
                                               const float* v_scale, int num_blocks,
                                               const int32_t* block_tables,
                                               int64_t block_table_stride, int max_blocks_per_seq,
                                               const int32_t* context_lens, int n_seqs,
                                               int n_q_heads, int n_kv_heads, int head_dim,
                                               int block_size, float scale, int dtype,
                                               void* workspace, size_t workspace_bytes,
                                               int* err_flags, pkv_stream_t stream,
                                               const void* schedule) {
  if (n_seqs < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!context_lens || !k_scale || !v_scale) return PKV_ERR_NULL_POINTER;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  a.n_seqs = n_seqs;
  a.n_tokens = n_seqs;
  a.max_query_len = 1;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  a.schedule = schedule;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  return decode_dispatch(a, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

static int pkv_paged_decode_append_attention_impl(void* out, int64_t out_row_stride, const void* q,
                                                  int64_t q_row_stride, const void* k_new,
                                                  const void* v_new, int64_t k_new_row_stride,
                                                  int64_t v_new_row_stride, void* k_pool,
                                                  void* v_pool, int num_blocks,
                                                  const int32_t* block_tables,
                                                  int64_t block_table_stride,
                                                  int max_blocks_per_seq,
                                                  const int32_t* context_lens, int n_seqs,
                                                  int n_q_heads, int n_kv_heads, int head_dim,
                                                  int block_size, float scale, int dtype,
                                                  void* workspace, size_t workspace_bytes,
                                                  int* err_flags, pkv_stream_t stream,
                                                  const void* schedule,
                                                  const int* input_ready = nullptr,
                                                  const LayerChain* chain = nullptr) {
  if (n_seqs < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!context_lens || !k_new || !v_new) return PKV_ERR_NULL_POINTER;
  if (input_ready && (reinterpret_cast<uintptr_t>(input_ready) & 3) != 0) return PKV_ERR_MISALIGNED;
  const int64_t kv_row = static_cast<int64_t>(n_kv_heads) * head_dim;
  if (k_new_row_stride < kv_row || v_new_row_stride < kv_row) return PKV_ERR_BAD_SHAPE;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  a.n_seqs = n_seqs;
  a.n_tokens = n_seqs;
  a.max_query_len = 1;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  a.schedule = schedule;
  a.k_new = k_new;
  a.v_new = v_new;
  a.k_new_stride = k_new_row_stride;
  a.v_new_stride = v_new_row_stride;
  a.input_ready = input_ready;
  a.chain = chain;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool fast = g_decode_impl.load() == PKV_DECODE_AUTO && decode_fast_supported(a);
  // only the tensor-core kernel waits on a word or chains layers
  if ((input_ready || chain) && !fast) return PKV_ERR_UNSUPPORTED;
  if (fast) {
    if (!workspace) return PKV_ERR_NULL_POINTER;
    if (workspace_bytes < decode_workspace_bytes(n_seqs, n_q_heads, head_dim))
      return PKV_ERR_WORKSPACE_TOO_SMALL;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return PKV_ERR_MISALIGNED;
    CUtensorMap km, vm;
    rc = cached_pool_map(&km, k_pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
    if (rc != 0) return rc;
    rc = cached_pool_map(&vm, v_pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
    if (rc != 0) return rc;
    return status_of(launch_decode_fast(a, &km, &vm, workspace, st));
  }
  // separate append (slot from the block table) + CUDA-core attention
  cudaError_t e = launch_append_at_context_end(k_new, v_new, k_new_row_stride, v_new_row_stride,
                                               k_pool, v_pool, block_tables, block_table_stride,
                                               max_blocks_per_seq, context_lens, n_seqs,
                                               num_blocks, block_size, n_kv_heads, head_dim,
                                               esize_of(dtype), err_flags, st);
  if (e != cudaSuccess) return status_of(e);
  a.k_new = a.v_new = nullptr;
  return status_of(launch_generic_attention(a, st));
}

static int pkv_paged_decode_append_attention_fp8_impl(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_new,
    const void* v_new, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pool,
    void* v_pool, float* k_scale, float* v_scale, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule, const LayerChain* chain = nullptr) {
  if (n_seqs < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!context_lens || !k_new || !v_new || !k_scale || !v_scale) return PKV_ERR_NULL_POINTER;
  const int64_t kv_row = static_cast<int64_t>(n_kv_heads) * head_dim;
  if (k_new_row_stride < kv_row || v_new_row_stride < kv_row) return PKV_ERR_BAD_SHAPE;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.context_lens = context_lens;
  a.n_seqs = n_seqs;
  a.n_tokens = n_seqs;
  a.max_query_len = 1;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  a.schedule = schedule;
  a.k_new = k_new;
  a.v_new = v_new;
  a.k_new_stride = k_new_row_stride;
  a.v_new_stride = v_new_row_stride;
  a.chain = chain;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (g_decode_impl.load() == PKV_DECODE_AUTO && decode_fast_supported(a))
    return decode_dispatch(a, workspace, workspace_bytes, st);
  if (chain) return PKV_ERR_UNSUPPORTED;  // only the tensor-core kernel chains layers
  // separate quantising append (slot from the block table) + CUDA-core attention
  cudaError_t e = launch_append_at_context_end_fp8(
      k_new, v_new, k_new_row_stride, v_new_row_stride, k_pool, v_pool, k_scale, v_scale,
      block_tables, block_table_stride, max_blocks_per_seq, context_lens, n_seqs, num_blocks,
      block_size, n_kv_heads, head_dim, dtype, err_flags, st);
  if (e != cudaSuccess) return status_of(e);
  a.k_new = a.v_new = nullptr;
  return decode_dispatch(a, workspace, workspace_bytes, st);
}

int pkv_paged_decode_append_attention_fp8(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_new,
    const void* v_new, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pool,
    void* v_pool, float* k_scale, float* v_scale, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream) {
  return pkv_paged_decode_append_attention_fp8_impl(
      out, out_row_stride, q, q_row_stride, k_new, v_new, k_new_row_stride, v_new_row_stride,
      k_pool, v_pool, k_scale, v_scale, num_blocks, block_tables, block_table_stride,
      max_blocks_per_seq, context_lens, n_seqs, n_q_heads, n_kv_heads, head_dim, block_size, scale,
      dtype, workspace, workspace_bytes, err_flags, stream, nullptr);
}

int pkv_paged_decode_append_attention_fp8_scheduled(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_new,
    const void* v_new, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pool,
    void* v_pool, float* k_scale, float* v_scale, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule) {
  if (!schedule) return PKV_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(schedule) & 15) != 0) return PKV_ERR_MISALIGNED;
  return pkv_paged_decode_append_attention_fp8_impl(
      out, out_row_stride, q, q_row_stride, k_new, v_new, k_new_row_stride, v_new_row_stride,
      k_pool, v_pool, k_scale, v_scale, num_blocks, block_tables, block_table_stride,
      max_blocks_per_seq, context_lens, n_seqs, n_q_heads, n_kv_heads, head_dim, block_size, scale,
      dtype, workspace, workspace_bytes, err_flags, stream, schedule);
}

int pkv_paged_decode_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                               const void* k_pool, const void* v_pool, int num_blocks,
                               const int32_t* block_tables, int64_t block_table_stride,
                               int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
                               int n_q_heads, int n_kv_heads, int head_dim, int block_size,
                               float scale, int dtype, void* workspace, size_t workspace_bytes,
                               int* err_flags, pkv_stream_t stream) {
  return pkv_paged_decode_attention_impl(out, out_row_stride, q, q_row_stride, k_pool, v_pool,
                                         num_blocks, block_tables, block_table_stride,
                                         max_blocks_per_seq, context_lens, n_seqs, n_q_heads,
                                         n_kv_heads, head_dim, block_size, scale, dtype, workspace,
                                         workspace_bytes, err_flags, stream, nullptr);
}

int pkv_paged_decode_attention_scheduled(void* out, int64_t out_row_stride, const void* q,
                                         int64_t q_row_stride, const void* k_pool,
                                         const void* v_pool, int num_blocks,
                                         const int32_t* block_tables, int64_t block_table_stride,
                                         int max_blocks_per_seq, const int32_t* context_lens,
                                         int n_seqs, int n_q_heads, int n_kv_heads, int head_dim,
                                         int block_size, float scale, int dtype, void* workspace,
                                         size_t workspace_bytes, int* err_flags,
                                         pkv_stream_t stream, const void* schedule) {
  if (!schedule) return PKV_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(schedule) & 15) != 0) return PKV_ERR_MISALIGNED;
  return pkv_paged_decode_attention_impl(out, out_row_stride, q, q_row_stride, k_pool, v_pool,
                                         num_blocks, block_tables, block_table_stride,
                                         max_blocks_per_seq, context_lens, n_seqs, n_q_heads,
                                         n_kv_heads, head_dim, block_size, scale, dtype, workspace,
                                         workspace_bytes, err_flags, stream, schedule);
}

int pkv_paged_decode_attention_fp8(void* out, int64_t out_row_stride, const void* q,
                                   int64_t q_row_stride, const void* k_pool, const void* v_pool,
                                   const float* k_scale, const float* v_scale, int num_blocks,
                                   const int32_t* block_tables, int64_t block_table_stride,
                                   int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
                                   int n_q_heads, int n_kv_heads, int head_dim, int block_size,
                                   float scale, int dtype, void* workspace, size_t workspace_bytes,
                                   int* err_flags, pkv_stream_t stream) {
  return pkv_paged_decode_attention_fp8_impl(out, out_row_stride, q, q_row_stride, k_pool, v_pool,
                                             k_scale, v_scale, num_blocks, block_tables,
                                             block_table_stride, max_blocks_per_seq, context_lens,
                                             n_seqs, n_q_heads, n_kv_heads, head_dim, block_size,
                                             scale, dtype, workspace, workspace_bytes, err_flags,
                                             stream, nullptr);
}

int pkv_paged_decode_attention_fp8_scheduled(void* out, int64_t out_row_stride, const void* q,
                                             int64_t q_row_stride, const void* k_pool,
                                             const void* v_pool, const float* k_scale,
                                             const float* v_scale, int num_blocks,
                                             const int32_t* block_tables,
                                             int64_t block_table_stride, int max_blocks_per_seq,
                                             const int32_t* context_lens, int n_seqs, int n_q_heads,
                                             int n_kv_heads, int head_dim, int block_size,
                                             float scale, int dtype, void* workspace,
                                             size_t workspace_bytes, int* err_flags,
                                             pkv_stream_t stream, const void* schedule) {
  if (!schedule) return PKV_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(schedule) & 15) != 0) return PKV_ERR_MISALIGNED;
  return pkv_paged_decode_attention_fp8_impl(out, out_row_stride, q, q_row_stride, k_pool, v_pool,
                                             k_scale, v_scale, num_blocks, block_tables,
                                             block_table_stride, max_blocks_per_seq, context_lens,
                                             n_seqs, n_q_heads, n_kv_heads, head_dim, block_size,
                                             scale, dtype, workspace, workspace_bytes, err_flags,
                                             stream, schedule);
}

int pkv_paged_decode_append_attention(void* out, int64_t out_row_stride, const void* q,
                                      int64_t q_row_stride, const void* k_new, const void* v_new,
                                      int64_t k_new_row_stride, int64_t v_new_row_stride,
                                      void* k_pool, void* v_pool, int num_blocks,
                                      const int32_t* block_tables, int64_t block_table_stride,
                                      int max_blocks_per_seq, const int32_t* context_lens,
                                      int n_seqs, int n_q_heads, int n_kv_heads, int head_dim,
                                      int block_size, float scale, int dtype, void* workspace,
                                      size_t workspace_bytes, int* err_flags, pkv_stream_t stream) {
  return pkv_paged_decode_append_attention_impl(out, out_row_stride, q, q_row_stride, k_new, v_new,
                                                k_new_row_stride, v_new_row_stride, k_pool, v_pool,
                                                num_blocks, block_tables, block_table_stride,
                                                max_blocks_per_seq, context_lens, n_seqs, n_q_heads,
                                                n_kv_heads, head_dim, block_size, scale, dtype,
                                                workspace, workspace_bytes, err_flags, stream,
                                                nullptr);
}

int pkv_paged_decode_append_attention_scheduled(void* out, int64_t out_row_stride, const void* q,
                                                int64_t q_row_stride, const void* k_new,
                                                const void* v_new, int64_t k_new_row_stride,
                                                int64_t v_new_row_stride, void* k_pool,
                                                void* v_pool, int num_blocks,
                                                const int32_t* block_tables,
                                                int64_t block_table_stride, int max_blocks_per_seq,
                                                const int32_t* context_lens, int n_seqs,
                                                int n_q_heads, int n_kv_heads, int head_dim,
                                                int block_size, float scale, int dtype,
                                                void* workspace, size_t workspace_bytes,
                                                int* err_flags, pkv_stream_t stream,
                                                const void* schedule) {
  if (!schedule) return PKV_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(schedule) & 15) != 0) return PKV_ERR_MISALIGNED;
  return pkv_paged_decode_append_attention_impl(out, out_row_stride, q, q_row_stride, k_new, v_new,
                                                k_new_row_stride, v_new_row_stride, k_pool, v_pool,
                                                num_blocks, block_tables, block_table_stride,
                                                max_blocks_per_seq, context_lens, n_seqs, n_q_heads,
                                                n_kv_heads, head_dim, block_size, scale, dtype,
                                                workspace, workspace_bytes, err_flags, stream,
                                                schedule);
}

int pkv_paged_decode_append_attention_layers(
    int n_layers, void* out, int64_t out_layer_stride, int64_t out_row_stride, const void* q,
    int64_t q_layer_stride, int64_t q_row_stride, const void* k_new, const void* v_new,
    int64_t new_layer_stride, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pools,
    void* v_pools, int64_t pool_layer_stride_bytes, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule, const int32_t* input_ready) {
  return pkv_paged_decode_append_attention_layers_flags(
      n_layers, out, out_layer_stride, out_row_stride, q, q_layer_stride, q_row_stride, k_new, v_new,
      new_layer_stride, k_new_row_stride, v_new_row_stride, k_pools, v_pools, pool_layer_stride_bytes,
      num_blocks, block_tables, block_table_stride, max_blocks_per_seq, context_lens, n_seqs,
      n_q_heads, n_kv_heads, head_dim, block_size, scale, dtype, workspace, workspace_bytes,
      err_flags, stream, schedule, input_ready, 0);
}

int pkv_paged_decode_append_attention_layers_flags(
    int n_layers, void* out, int64_t out_layer_stride, int64_t out_row_stride, const void* q,
    int64_t q_layer_stride, int64_t q_row_stride, const void* k_new, const void* v_new,
    int64_t new_layer_stride, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pools,
    void* v_pools, int64_t pool_layer_stride_bytes, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule, const int32_t* input_ready, int flags) {
  if ((flags & ~PKV_LAYERS_DEFER_FIRST) != 0) return PKV_ERR_UNSUPPORTED;
  const bool defer_first = (flags & PKV_LAYERS_DEFER_FIRST) != 0;
  if (n_layers < 0 || n_seqs < 0) return PKV_ERR_BAD_SHAPE;
  if (n_layers == 0 || n_seqs == 0) return PKV_OK;
  if (!out || !q || !k_new || !v_new || !k_pools || !v_pools) return PKV_ERR_NULL_POINTER;
  if (schedule && (reinterpret_cast<uintptr_t>(schedule) & 15) != 0) return PKV_ERR_MISALIGNED;
  if (dtype != PKV_DTYPE_F32 && dtype != PKV_DTYPE_F16 && dtype != PKV_DTYPE_BF16)
    return PKV_ERR_BAD_DTYPE;
  const int64_t es = esize_of(dtype);
  // consecutive layers' pools must not overlap
  const int64_t pool_bytes = static_cast<int64_t>(num_blocks) * block_size * n_kv_heads *
                             head_dim * es;
  if (n_layers > 1 && (pool_layer_stride_bytes < pool_bytes || out_layer_stride <= 0 ||
                       q_layer_stride <= 0 || new_layer_stride <= 0))
    return PKV_ERR_BAD_SHAPE;
  if ((pool_layer_stride_bytes & 15) != 0) return PKV_ERR_MISALIGNED;
  auto at = [](const void* base, int64_t off_bytes) {
    return static_cast<const void*>(static_cast<const uint8_t*>(base) + off_bytes);
  };
  auto layer_call = [&](int l) -> int {
    void* o = const_cast<void*>(at(out, l * out_layer_stride * es));
    const void* ql = at(q, l * q_layer_stride * es);
    const void* kn = at(k_new, l * new_layer_stride * es);
    const void* vn = at(v_new, l * new_layer_stride * es);
    void* kp = const_cast<void*>(at(k_pools, l * pool_layer_stride_bytes));
    void* vp = const_cast<void*>(at(v_pools, l * pool_layer_stride_bytes));
    return pkv_paged_decode_append_attention_impl(
        o, out_row_stride, ql, q_row_stride, kn, vn, k_new_row_stride, v_new_row_stride, kp, vp,
        num_blocks, block_tables, block_table_stride, max_blocks_per_seq, context_lens, n_seqs,
        n_q_heads, n_kv_heads, head_dim, block_size, scale, dtype, workspace, workspace_bytes,
        err_flags, stream, schedule, input_ready ? input_ready + l : nullptr);
  };
  // the shared arguments and the last layer's pointers are checked before
  // the first launch, so a bad call issues nothing
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pools, v_pools, num_blocks,
                      block_tables, block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads,
                      head_dim, block_size, dtype);
  if (rc != PKV_OK) return rc;
  const int last = n_layers - 1;
  rc = check_attn(at(out, last * out_layer_stride * es), out_row_stride,
                  at(q, last * q_layer_stride * es), q_row_stride,
                  at(k_pools, last * pool_layer_stride_bytes),
                  at(v_pools, last * pool_layer_stride_bytes), num_blocks, block_tables,
                  block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                  block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!context_lens) return PKV_ERR_NULL_POINTER;
  // A workspace of one split-K set per layer chains the layers: the decode
  // kernels run back to back, each later one waiting for its predecessor only
  // at its end (so it starts on the SMs the previous layer's tail frees), and
  // one merge launch covers every layer at the end.  Otherwise each layer's
  // decode is followed by its own merge.
  // PKV_LAYERS_DEFER_FIRST: the first layer's decode defers its wait too
  // (the caller's promise that nothing still running before the call touches
  // what the call reads or writes), also for a single layer.
  const size_t ws1 = decode_workspace_bytes(n_seqs, n_q_heads, head_dim);
  if ((n_layers > 1 || defer_first) && workspace && ws1 > 0 &&
      workspace_bytes / static_cast<size_t>(n_layers) >= ws1) {
    LayerChain ch{0, 0, n_layers, out, out_layer_stride, workspace, static_cast<int64_t>(ws1)};
    for (int l = 0; l < n_layers; ++l) {
      ch.defer_wait = l > 0 || defer_first;
      ch.merge = l == n_layers - 1;
      void* o = const_cast<void*>(at(out, l * out_layer_stride * es));
      void* wsl = static_cast<uint8_t*>(workspace) + static_cast<size_t>(l) * ws1;
      rc = pkv_paged_decode_append_attention_impl(
          o, out_row_stride, at(q, l * q_layer_stride * es), q_row_stride,
          at(k_new, l * new_layer_stride * es), at(v_new, l * new_layer_stride * es), k_new_row_stride,
          v_new_row_stride, const_cast<void*>(at(k_pools, l * pool_layer_stride_bytes)),
          const_cast<void*>(at(v_pools, l * pool_layer_stride_bytes)), num_blocks, block_tables,
          block_table_stride, max_blocks_per_seq, context_lens, n_seqs, n_q_heads, n_kv_heads,
          head_dim, block_size, scale, dtype, wsl, ws1, err_flags, stream, schedule,
          input_ready ? input_ready + l : nullptr, &ch);
      if (rc == PKV_ERR_UNSUPPORTED && l == 0 && !input_ready) break;  // not the tensor-core path
      if (rc != PKV_OK) return rc;
      if (l == n_layers - 1) return PKV_OK;
    }
  }
  for (int l = 0; l < n_layers; ++l) {
    rc = layer_call(l);
    if (rc != PKV_OK) return rc;
  }
  return PKV_OK;
}

int pkv_paged_decode_append_attention_fp8_layers(
    int n_layers, void* out, int64_t out_layer_stride, int64_t out_row_stride, const void* q,
    int64_t q_layer_stride, int64_t q_row_stride, const void* k_new, const void* v_new,
    int64_t new_layer_stride, int64_t k_new_row_stride, int64_t v_new_row_stride, void* k_pools,
    void* v_pools, int64_t pool_layer_stride_bytes, float* k_scales, float* v_scales,
    int64_t scale_layer_stride, int num_blocks, const int32_t* block_tables,
    int64_t block_table_stride, int max_blocks_per_seq, const int32_t* context_lens, int n_seqs,
    int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale, int dtype,
    void* workspace, size_t workspace_bytes, int* err_flags, pkv_stream_t stream,
    const void* schedule) {
  if (n_layers < 0 || n_seqs < 0) return PKV_ERR_BAD_SHAPE;
  if (n_layers == 0 || n_seqs == 0) return PKV_OK;
  if (!out || !q || !k_new || !v_new || !k_pools || !v_pools || !k_scales || !v_scales || !context_lens)
    return PKV_ERR_NULL_POINTER;
  if (schedule && (reinterpret_cast<uintptr_t>(schedule) & 15) != 0) return PKV_ERR_MISALIGNED;
  if (dtype != PKV_DTYPE_F16 && dtype != PKV_DTYPE_BF16) return PKV_ERR_BAD_DTYPE;
  const int64_t es = esize_of(dtype);
  const int64_t pool_bytes = static_cast<int64_t>(num_blocks) * block_size * n_kv_heads * head_dim;
  const int64_t scale_count = static_cast<int64_t>(num_blocks) * block_size * n_kv_heads;
  if (n_layers > 1 && (pool_layer_stride_bytes < pool_bytes || scale_layer_stride < scale_count ||
                       out_layer_stride <= 0 || q_layer_stride <= 0 || new_layer_stride <= 0))
    return PKV_ERR_BAD_SHAPE;
  if ((pool_layer_stride_bytes & 15) != 0 || (scale_layer_stride & 3) != 0) return PKV_ERR_MISALIGNED;
  auto at = [](const void* base, int64_t off_bytes) {
    return static_cast<const void*>(static_cast<const uint8_t*>(base) + off_bytes);
  };
  // layer l's call; `chain`: the call's layers chain (a split-K set per layer)
  auto layer_call = [&](int l, const LayerChain* chain, void* ws, size_t wsb) -> int {
    return pkv_paged_decode_append_attention_fp8_impl(
        const_cast<void*>(at(out, l * out_layer_stride * es)), out_row_stride,
        at(q, l * q_layer_stride * es), q_row_stride, at(k_new, l * new_layer_stride * es),
        at(v_new, l * new_layer_stride * es), k_new_row_stride, v_new_row_stride,
        const_cast<void*>(at(k_pools, l * pool_layer_stride_bytes)),
        const_cast<void*>(at(v_pools, l * pool_layer_stride_bytes)), k_scales + l * scale_layer_stride,
        v_scales + l * scale_layer_stride, num_blocks, block_tables, block_table_stride,
        max_blocks_per_seq, context_lens, n_seqs, n_q_heads, n_kv_heads, head_dim, block_size, scale,
        dtype, ws, wsb, err_flags, stream, schedule, chain);
  };
  // the first and the last layer's pointers are checked before anything launches
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pools, v_pools, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  const int last = n_layers - 1;
  rc = check_attn(at(out, last * out_layer_stride * es), out_row_stride, at(q, last * q_layer_stride * es),
                  q_row_stride, at(k_pools, last * pool_layer_stride_bytes),
                  at(v_pools, last * pool_layer_stride_bytes), num_blocks, block_tables,
                  block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim, block_size,
                  dtype);
  if (rc != PKV_OK) return rc;
  // a split-K set per layer chains the layers, as in the 16-bit call
  const size_t ws1 = decode_workspace_bytes(n_seqs, n_q_heads, head_dim);
  if (n_layers > 1 && workspace && ws1 > 0 && workspace_bytes / static_cast<size_t>(n_layers) >= ws1) {
    LayerChain ch{0, 0, n_layers, out, out_layer_stride, workspace, static_cast<int64_t>(ws1)};
    for (int l = 0; l < n_layers; ++l) {
      ch.defer_wait = l > 0;
      ch.merge = l == last;
      rc = layer_call(l, &ch, static_cast<uint8_t*>(workspace) + static_cast<size_t>(l) * ws1, ws1);
      if (rc == PKV_ERR_UNSUPPORTED && l == 0) break;  // not the tensor-core path
      if (rc != PKV_OK) return rc;
      if (l == last) return PKV_OK;
    }
  }
  for (int l = 0; l < n_layers; ++l) {
    rc = layer_call(l, nullptr, workspace, workspace_bytes);
    if (rc != PKV_OK) return rc;
  }
  return PKV_OK;
}

// the tcgen05 prefill over fp8 pools, e4m3 tiles converted inside the kernel
static int prefill_fp8_tc(const AttnArgs& a, cudaStream_t st) {
  CUtensorMap qm, km, vm;
  int rc = encode_q_tensormap(&qm, a.q, a.q_stride, a.n_tokens, a.n_q_heads, a.head_dim, a.dtype);
  if (rc != 0) return rc;
  rc = cached_pool_map(&km, a.k_pool, a.num_blocks, a.block_size, a.n_kv_heads, a.head_dim, kPoolFp8);
  if (rc != 0) return rc;
  rc = cached_pool_map(&vm, a.v_pool, a.num_blocks, a.block_size, a.n_kv_heads, a.head_dim, kPoolFp8);
  if (rc != 0) return rc;
  return status_of(launch_prefill_fast(a, &qm, &km, &vm, st));
}

int pkv_paged_prefill_attention_fp8_tc(void* out, int64_t out_row_stride, const void* q,
                                       int64_t q_row_stride, const void* k_pool, const void* v_pool,
                                       const float* k_scale, const float* v_scale, int num_blocks,
                                       const int32_t* block_tables, int64_t block_table_stride,
                                       int max_blocks_per_seq, const int32_t* query_start_loc,
                                       const int32_t* num_prior, int n_seqs, int n_tokens,
                                       int max_query_len, int n_q_heads, int n_kv_heads,
                                       int head_dim, int block_size, float scale, int dtype,
                                       int* err_flags, pkv_stream_t stream) {
  if (n_seqs < 0 || n_tokens < 0 || max_query_len < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0 || n_tokens == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!query_start_loc || !num_prior || !k_scale || !v_scale) return PKV_ERR_NULL_POINTER;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.query_start_loc = query_start_loc;
  a.num_prior = num_prior;
  a.n_seqs = n_seqs;
  a.n_tokens = n_tokens;
  a.max_query_len = max_query_len;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  if (!prefill_fp8_tc_supported(a)) return PKV_ERR_UNSUPPORTED;
  return prefill_fp8_tc(a, static_cast<cudaStream_t>(stream));
}

size_t pkv_prefill_fp8_scratch_bytes(int n_seqs, int max_blocks_per_seq, int n_kv_heads,
                                     int head_dim) {
  if (n_seqs < 0 || max_blocks_per_seq < 0 || n_kv_heads <= 0 || head_dim <= 0) return 0;
  return prefill_fp8_scratch_bytes(n_seqs, max_blocks_per_seq, n_kv_heads, head_dim);
}

int pkv_paged_prefill_attention_fp8_scratch(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_pool,
    const void* v_pool, const float* k_scale, const float* v_scale, int num_blocks,
    const int32_t* block_tables, int64_t block_table_stride, int max_blocks_per_seq,
    const int32_t* query_start_loc, const int32_t* num_prior, int n_seqs, int n_tokens,
    int max_query_len, int n_q_heads, int n_kv_heads, int head_dim, int block_size, float scale,
    int dtype, void* scratch, size_t scratch_bytes, int* err_flags, pkv_stream_t stream) {
  if (n_seqs < 0 || n_tokens < 0 || max_query_len < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0 || n_tokens == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!query_start_loc || !num_prior || !k_scale || !v_scale || !scratch) return PKV_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(scratch) & 255) != 0) return PKV_ERR_MISALIGNED;
  if (scratch_bytes < prefill_fp8_scratch_bytes(n_seqs, max_blocks_per_seq, n_kv_heads, head_dim))
    return PKV_ERR_WORKSPACE_TOO_SMALL;
  if (n_seqs > 65535) return PKV_ERR_UNSUPPORTED;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.query_start_loc = query_start_loc;
  a.num_prior = num_prior;
  a.n_seqs = n_seqs;
  a.n_tokens = n_tokens;
  a.max_query_len = max_query_len;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  AttnArgs t = a;  // the tensor-core prefill over the 16-bit scratch pool
  t.k_scale = t.v_scale = nullptr;
  t.k_pool = t.v_pool = scratch;  // alignment stand-ins until the pass sets them
  // the pass reads the e4m3 pools 16 bytes at a time
  const bool pools16 = ((reinterpret_cast<uintptr_t>(k_pool) | reinterpret_cast<uintptr_t>(v_pool)) & 15) == 0;
  if (g_decode_impl.load() != PKV_DECODE_AUTO || !prefill_fast_supported(t) || !pools16)
    return status_of(launch_generic_attention(a, st));
  void *kq = nullptr, *vq = nullptr;
  int32_t* tab = nullptr;
  cudaError_t e = launch_dequant_blocks(a, scratch, st, &kq, &vq, &tab);
  if (e != cudaSuccess) return status_of(e);
  t.k_pool = kq;
  t.v_pool = vq;
  t.num_blocks = n_seqs * max_blocks_per_seq;
  t.block_tables = tab;
  t.bt_stride = max_blocks_per_seq;
  CUtensorMap qm, km, vm;
  rc = encode_q_tensormap(&qm, q, q_row_stride, n_tokens, n_q_heads, head_dim, dtype);
  if (rc != 0) return rc;
  // the scratch pool's maps are encoded per call (its block count follows the step)
  rc = encode_pool_tensormap(&km, kq, t.num_blocks, block_size, n_kv_heads, head_dim, dtype);
  if (rc != 0) return rc;
  rc = encode_pool_tensormap(&vm, vq, t.num_blocks, block_size, n_kv_heads, head_dim, dtype);
  if (rc != 0) return rc;
  return status_of(launch_prefill_fast(t, &qm, &km, &vm, st));
}

int pkv_paged_prefill_attention(void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride,
                                const void* k_pool, const void* v_pool, int num_blocks,
                                const int32_t* block_tables, int64_t block_table_stride,
                                int max_blocks_per_seq, const int32_t* query_start_loc,
                                const int32_t* num_prior, int n_seqs, int n_tokens, int max_query_len,
                                int n_q_heads, int n_kv_heads, int head_dim, int block_size,
                                float scale, int dtype, int* err_flags, pkv_stream_t stream) {
  if (n_seqs < 0 || n_tokens < 0 || max_query_len < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0 || n_tokens == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!query_start_loc || !num_prior) return PKV_ERR_NULL_POINTER;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.query_start_loc = query_start_loc;
  a.num_prior = num_prior;
  a.n_seqs = n_seqs;
  a.n_tokens = n_tokens;
  a.max_query_len = max_query_len;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (g_decode_impl.load() == PKV_DECODE_AUTO && prefill_fast_supported(a)) {
    CUtensorMap qm, km, vm;
    rc = encode_q_tensormap(&qm, q, q_row_stride, n_tokens, n_q_heads, head_dim, dtype);
    if (rc != 0) return rc;
    rc = cached_pool_map(&km, k_pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
    if (rc != 0) return rc;
    rc = cached_pool_map(&vm, v_pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
    if (rc != 0) return rc;
    return status_of(launch_prefill_fast(a, &qm, &km, &vm, st));
  }
  return status_of(launch_generic_attention(a, st));
}

int pkv_paged_prefill_attention_fp8(void* out, int64_t out_row_stride, const void* q,
                                    int64_t q_row_stride, const void* k_pool, const void* v_pool,
                                    const float* k_scale, const float* v_scale, int num_blocks,
                                    const int32_t* block_tables, int64_t block_table_stride,
                                    int max_blocks_per_seq, const int32_t* query_start_loc,
                                    const int32_t* num_prior, int n_seqs, int n_tokens,
                                    int max_query_len, int n_q_heads, int n_kv_heads, int head_dim,
                                    int block_size, float scale, int dtype, int* err_flags,
                                    pkv_stream_t stream) {
  if (n_seqs < 0 || n_tokens < 0 || max_query_len < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0 || n_tokens == 0) return PKV_OK;
  int rc = check_attn(out, out_row_stride, q, q_row_stride, k_pool, v_pool, num_blocks, block_tables,
                      block_table_stride, max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
                      block_size, dtype);
  if (rc != PKV_OK) return rc;
  if (!query_start_loc || !num_prior || !k_scale || !v_scale) return PKV_ERR_NULL_POINTER;
  AttnArgs a{};
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.k_pool = k_pool;
  a.v_pool = v_pool;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.query_start_loc = query_start_loc;
  a.num_prior = num_prior;
  a.n_seqs = n_seqs;
  a.n_tokens = n_tokens;
  a.max_query_len = max_query_len;
  a.n_q_heads = n_q_heads;
  a.n_kv_heads = n_kv_heads;
  a.head_dim = head_dim;
  a.block_size = block_size;
  a.scale = scale;
  a.dtype = dtype;
  a.err = err_flags;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  // the CUDA-core kernel (dequantise on load); the tensor-core prefill reads
  // 16-bit pools only
  return status_of(launch_generic_attention(a, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
