// pkv_prefill_fp8.cu -- chunked prefill over fp8 e4m3 pools on the tensor cores.
//
// The tcgen05 prefill kernel (pkv_prefill.cu) reads 16-bit K/V tiles by TMA.
// For fp8 pools, one pass first writes the blocks the step's sequences can
// see into a caller-provided 16-bit scratch pool: value = e4m3(byte) x the
// row's fp32 scale, rounded once to the query dtype.  Then the unchanged
// tcgen05 kernel runs over that pool through an identity block table (block
// j of sequence s sits at scratch block s * max_blocks + j).  For the
// config-4 shape (16 chunks of 512 queries over priors of up to 4 K tokens)
// the pass moves about 3 bytes per KV element (one read, two written); the
// prefill reads the 16-bit scratch (about 21 MB, well inside the 126 MB L2)
// right after it.
//
// Replaces, for fp8 pools, the gather + _attention of the reference for
// num_new > 1 (mini_engine/paged/block_manager.py:136-141,
// mini_engine/model/qwen2.py:98-128).
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

namespace {

constexpr int kDqThreads = 256;

// CTA (j, s): block j of sequence s, K and V.  Each thread converts 16
// consecutive bytes of one (row, KV head): one 16-byte load, eight e4m3x2 ->
// f16x2 conversions, the row's fp32 scale, two 16-byte stores.  The rows past
// the sequence's visible keys (num_prior + its chunk) are written as zeros,
// so the scratch holds no stale bytes the prefill kernel could multiply by a
// zero probability.  Launched with programmatic serialization: nothing is
// read or written before the wait (the append before it writes the pools,
// and the prefill of the previous layer may still read the scratch), and
// each CTA then triggers the prefill after it, whose set-up overlaps this
// pass's tail.  (Four blocks per CTA with four loads in flight per thread
// measured slower: fewer CTAs hide less latency.)
template <typename T>
__global__ void __launch_bounds__(kDqThreads) dequant_blocks_kernel(
    const uint8_t* __restrict__ k_pool, const uint8_t* __restrict__ v_pool,
    const float* __restrict__ k_scale, const float* __restrict__ v_scale,
    const int32_t* __restrict__ tables, int64_t bt_stride, int max_blocks,
    const int32_t* __restrict__ qsl, const int32_t* __restrict__ num_prior, int num_blocks,
    int hkv, T* __restrict__ k_out, T* __restrict__ v_out, int32_t* __restrict__ table_out,
    int* err) {
  pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
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
  const int per = 16 * hkv * 4;  // 16-byte chunks of one tensor's block (head_dim 64)
  const int valid = keys - j * 16;  // rows of this block that are keys
  for (int c = threadIdx.x; c < 2 * per; c += kDqThreads) {
    const bool isv = c >= per;
    const int cc = isv ? c - per : c;
    const int row = cc / (hkv * 4), h = (cc >> 2) - row * hkv;
    uint4 o0 = make_uint4(0u, 0u, 0u, 0u), o1 = o0;
    if (!bad && row < valid) {
      const int64_t src = static_cast<int64_t>(blk) * (per * 16) + cc * 16;
      const uint4 w = *reinterpret_cast<const uint4*>((isv ? v_pool : k_pool) + src);
      const float sc = (isv ? v_scale : k_scale)[(static_cast<int64_t>(blk) * 16 + row) * hkv + h];
      const uint32_t in[4] = {w.x, w.y, w.z, w.w};
      uint32_t o[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // bytes (0, 1) and (2, 3) of the word: exact fp16, then x scale in
        // fp32 and one rounding to T (as fp8_to_float(b) * scale)
        const __half2_raw lo =
            __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(in[k] & 0xffffu), __NV_E4M3);
        const __half2_raw hi =
            __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(in[k] >> 16), __NV_E4M3);
        const float2 fl = __half22float2(__half2(lo));
        const float2 fh = __half22float2(__half2(hi));
        o[2 * k] = pack2<T>(fl.x * sc, fl.y * sc);
        o[2 * k + 1] = pack2<T>(fh.x * sc, fh.y * sc);
      }
      o0 = make_uint4(o[0], o[1], o[2], o[3]);
      o1 = make_uint4(o[4], o[5], o[6], o[7]);
    }
    uint4* dst = reinterpret_cast<uint4*>((isv ? v_out : k_out) + dst_blk * (per * 16) + cc * 16);
    dst[0] = o0;
    dst[1] = o1;
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
  if (a.head_dim != 64) return cudaErrorNotSupported;  // the tensor-core prefill's head_dim
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.max_blocks, a.n_seqs);
  cfg.blockDim = dim3(kDqThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto go = [&](auto tag) {
    using T = decltype(tag);
    return cudaLaunchKernelEx(&cfg, dequant_blocks_kernel<T>, static_cast<const uint8_t*>(a.k_pool),
                              static_cast<const uint8_t*>(a.v_pool), a.k_scale, a.v_scale,
                              a.block_tables, a.bt_stride, a.max_blocks, a.query_start_loc,
                              a.num_prior, a.num_blocks, a.n_kv_heads, static_cast<T*>(*k_out),
                              static_cast<T*>(*v_out), *table_out, a.err);
  };
  if (a.dtype == PKV_DTYPE_F16) return go(__half{});
  return go(__nv_bfloat16{});
}

}  // namespace pkv
