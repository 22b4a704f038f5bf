// pkv_prefill_fp8.cu -- chunked prefill over fp8 e4m3 pools on the tensor cores.
//
// The tcgen05 prefill kernel (pkv_prefill.cu) reads 16-bit K/V tiles by TMA.
// For fp8 pools, one pass first writes the blocks the step's sequences can
// see into a caller-provided 16-bit scratch pool: value = e4m3(byte) x the
// row's fp32 scale, rounded once to the query dtype.  Then the unchanged
// tcgen05 kernel runs over that pool through an identity block table (block
// j of sequence s sits at scratch block s * max_blocks + j).  For the
// BASELINE config-4 shape the pass moves about 3 bytes per KV element (one
// read, two written) against a prefill that is tensor-bound.
//
// Replaces, for fp8 pools, the gather + _attention of the reference for
// num_new > 1 (mini_engine/paged/block_manager.py:136-141,
// mini_engine/model/qwen2.py:98-128).
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

namespace {

constexpr int kDqThreads = 256;

// CTA (j, s): block j of sequence s.  The rows past the sequence's visible
// keys (num_prior + its chunk) are written as zeros, so the scratch holds no
// stale bytes the prefill kernel could multiply by a zero probability.
template <typename T>
__global__ void __launch_bounds__(kDqThreads) dequant_blocks_kernel(
    const uint8_t* __restrict__ k_pool, const uint8_t* __restrict__ v_pool,
    const float* __restrict__ k_scale, const float* __restrict__ v_scale,
    const int32_t* __restrict__ tables, int64_t bt_stride, int max_blocks,
    const int32_t* __restrict__ qsl, const int32_t* __restrict__ num_prior, int num_blocks,
    int hkv, int d, T* __restrict__ k_out, T* __restrict__ v_out, int32_t* __restrict__ table_out,
    int* err) {
  const int j = blockIdx.x, s = blockIdx.y;
  const int keys = num_prior[s] + (qsl[s + 1] - qsl[s]);
  const int used = min((keys + 15) / 16, max_blocks);
  if (keys > max_blocks * 16 && j == 0 && threadIdx.x == 0)
    raise_flag(err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
  const int64_t dst_blk = static_cast<int64_t>(s) * max_blocks + j;
  if (threadIdx.x == 0) table_out[dst_blk] = static_cast<int32_t>(dst_blk);
  if (j >= used) return;
  int blk = tables[static_cast<int64_t>(s) * bt_stride + j];
  const bool bad = blk < 0 || blk >= num_blocks;
  if (bad && threadIdx.x == 0) raise_flag(err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
  const int row_elems = hkv * d;
  const int elems = 16 * row_elems;
  const int valid = keys - j * 16;  // rows of this block that are keys
  for (int e = threadIdx.x * 4; e < elems; e += kDqThreads * 4) {
    const int row = e / row_elems, h = (e - row * row_elems) / d;
    float kv[4] = {0.f, 0.f, 0.f, 0.f}, vv[4] = {0.f, 0.f, 0.f, 0.f};
    if (!bad && row < valid) {
      const int64_t src = static_cast<int64_t>(blk) * elems + e;
      const uint32_t kb = *reinterpret_cast<const uint32_t*>(k_pool + src);
      const uint32_t vb = *reinterpret_cast<const uint32_t*>(v_pool + src);
      const int64_t srow = (static_cast<int64_t>(blk) * 16 + row) * hkv + h;
      const float ks = k_scale[srow], vs = v_scale[srow];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kv[i] = fp8_to_float(static_cast<uint8_t>(kb >> (8 * i))) * ks;
        vv[i] = fp8_to_float(static_cast<uint8_t>(vb >> (8 * i))) * vs;
      }
    }
    const int64_t dst = dst_blk * elems + e;
    *reinterpret_cast<uint2*>(k_out + dst) = make_uint2(pack2<T>(kv[0], kv[1]), pack2<T>(kv[2], kv[3]));
    *reinterpret_cast<uint2*>(v_out + dst) = make_uint2(pack2<T>(vv[0], vv[1]), pack2<T>(vv[2], vv[3]));
  }
}

}  // namespace

size_t prefill_fp8_scratch_bytes(int n_seqs, int max_blocks, int n_kv_heads, int head_dim) {
  const size_t blocks = static_cast<size_t>(n_seqs) * max_blocks;
  const size_t table = (blocks * 4 + 255) & ~static_cast<size_t>(255);
  const size_t pool = blocks * 16 * n_kv_heads * head_dim * 2;  // 16-bit elements
  return table + 2 * pool;
}

cudaError_t launch_dequant_blocks(const AttnArgs& a, void* scratch, cudaStream_t stream,
                                  void** k_out, void** v_out, int32_t** table_out) {
  const size_t blocks = static_cast<size_t>(a.n_seqs) * a.max_blocks;
  const size_t table = (blocks * 4 + 255) & ~static_cast<size_t>(255);
  const size_t pool = blocks * 16 * a.n_kv_heads * a.head_dim * 2;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  *table_out = reinterpret_cast<int32_t*>(base);
  *k_out = base + table;
  *v_out = base + table + pool;
  dim3 grid(a.max_blocks, a.n_seqs);
  auto go = [&](auto tag) {
    using T = decltype(tag);
    dequant_blocks_kernel<T><<<grid, kDqThreads, 0, stream>>>(
        static_cast<const uint8_t*>(a.k_pool), static_cast<const uint8_t*>(a.v_pool), a.k_scale,
        a.v_scale, a.block_tables, a.bt_stride, a.max_blocks, a.query_start_loc, a.num_prior,
        a.num_blocks, a.n_kv_heads, a.head_dim, static_cast<T*>(*k_out), static_cast<T*>(*v_out),
        *table_out, a.err);
    return cudaGetLastError();
  };
  if (a.dtype == PKV_DTYPE_F16) return go(__half{});
  return go(__nv_bfloat16{});
}

}  // namespace pkv
