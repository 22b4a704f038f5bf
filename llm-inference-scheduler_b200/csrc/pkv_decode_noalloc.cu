// pkv_decode_noalloc.cu -- paged decode attention without any device allocation.
//
// Some hosts of this library cannot allocate device memory where they run
// decode attention: a thin FFI layer that only forwards the pointers it was
// given, or a process whose GPU memory is fully owned by another allocator.
// They cannot hand pkv_paged_decode_attention its split-K workspace, so this
// file gives them pkv_paged_decode_attention_noalloc, which runs the same
// kernels with the partials kept in a fixed array compiled into the library's
// device image (PKV_NOALLOC_SCRATCH_BYTES per GPU, resident from module load
// until the process exits).  Nothing is allocated per call.
//
// The array's host-side name is only a handle: its device address is looked
// up with cudaGetSymbolAddress, with the device current, on the first call in
// each CUDA context, and cached under that context's unique id.  A context
// that is destroyed and made again (cudaDeviceReset, or the primary context
// released and retained again) reloads the module, so the array may move; the
// new context has a new id and the address is looked up again.  All calls on
// a device share the array; it keeps the last call's partials, none of which
// need to start at zero, and calls that overlap on the GPU race on it.
#include <cudaTypedefs.h>

#include <mutex>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {
namespace {

constexpr size_t kScratchBytes = PKV_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchSlot {
  unsigned long long ctx_id = 0;  // unique id of the context the address belongs to (0: none)
  void* addr = nullptr;
};
std::mutex g_scratch_mu;
ScratchSlot g_scratch[kMaxDevices];

PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_fns_once;

// Unique id of the calling thread's current context (0 when none is current).
int current_context_id(unsigned long long* id) {
  std::call_once(g_ctx_fns_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 4000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  });
  if (!g_ctx_current || !g_ctx_id) return PKV_ERR_DRIVER;
  CUcontext ctx = nullptr;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS) return PKV_ERR_DRIVER;
  *id = 0;
  if (ctx && g_ctx_id(ctx, id) != CUDA_SUCCESS) return PKV_ERR_DRIVER;
  return PKV_OK;
}

// Device address of g_decode_scratch in the current device's current context.
int scratch_on_current_device(void** addr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return PKV_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  unsigned long long id = 0;
  int rc = current_context_id(&id);
  if (rc != PKV_OK) return rc;
  ScratchSlot& slot = g_scratch[dev];
  if (id == 0 || slot.addr == nullptr || slot.ctx_id != id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);  // makes the primary context current if needed
    if (e != cudaSuccess) return static_cast<int>(e);
    rc = current_context_id(&id);
    if (rc != PKV_OK) return rc;
    slot.ctx_id = id;
    slot.addr = p;
  }
  *addr = slot.addr;
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_paged_decode_attention_noalloc(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, const void* k_pool,
    const void* v_pool, int num_blocks, const int32_t* block_tables, int64_t block_table_stride,
    int max_blocks_per_seq, const int32_t* context_lens, int n_seqs, int n_q_heads,
    int n_kv_heads, int head_dim, int block_size, float scale, int dtype, int* err_flags,
    pkv_stream_t stream) {
  if (n_seqs < 0) return PKV_ERR_BAD_SHAPE;
  if (n_seqs == 0) return PKV_OK;
  int rc = validate_attention_args(out, out_row_stride, q, q_row_stride, k_pool, v_pool,
                                   num_blocks, block_tables, block_table_stride,
                                   max_blocks_per_seq, n_q_heads, n_kv_heads, head_dim,
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
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (decode_impl_setting() == PKV_DECODE_AUTO && decode_fast_supported(a)) {
    if (decode_workspace_bytes(n_seqs, n_q_heads, head_dim) > kScratchBytes)
      return PKV_ERR_SCRATCH_LIMIT;
    void* scratch = nullptr;
    rc = scratch_on_current_device(&scratch);
    if (rc != PKV_OK) return rc;
    CUtensorMap km, vm;
    rc = pool_tensormap(&km, k_pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
    if (rc != 0) return rc;
    rc = pool_tensormap(&vm, v_pool, num_blocks, block_size, n_kv_heads, head_dim, dtype);
    if (rc != 0) return rc;
    const cudaError_t e = launch_decode_fast(a, &km, &vm, scratch, st);
    return e == cudaSuccess ? PKV_OK : static_cast<int>(e);
  }
  // the CUDA-core kernel keeps no split-K state: no scratch needed
  const cudaError_t e = launch_generic_attention(a, st);
  return e == cudaSuccess ? PKV_OK : static_cast<int>(e);
}
