// pkv_attention_generic.cu -- portable paged attention on CUDA cores.
//
// Serves every shape / dtype the tensor-core kernels do not: fp32 KV (the
// reference's default CPU dtype), head_dim other than 64, other block sizes
// and GQA ratios.  One warp per (query row, q head); keys are visited 32 at a
// time (lane = key) with an fp32 online softmax, and the PV product keeps
// head_dim/32 output dims per lane.  Semantics follow the reference's gather
// + _attention (mini_engine/paged/block_manager.py:136-141,
// mini_engine/model/qwen2.py:98-128): key j is visible to new token i of a
// sequence iff j <= num_prior + i.  With fp8 e4m3 pools (AttnArgs::k_scale
// set) every K/V element is dequantised as e4m3(byte) * scale of its (slot,
// KV head) row before it enters the fp32 arithmetic.
#include <float.h>

#include <type_traits>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

constexpr int kGenericWarps = 4;
constexpr int kGenericMaxDPerLane = 8;  // head_dim <= 256

// K/V element d of pool row `row` (slot * n_kv_heads + head), as fp32
template <typename T, bool FP8>
__device__ __forceinline__ float kv_elem(const void* pool, const float* scales, int64_t row,
                                         int D, int d) {
  if constexpr (FP8) {
    return fp8_to_float(static_cast<const uint8_t*>(pool)[row * D + d]) * __ldg(scales + row);
  } else {
    return Elem<T>::to_f(static_cast<const T*>(pool)[row * D + d]);
  }
}

template <typename T, bool FP8>
__global__ void __launch_bounds__(kGenericWarps * 32) generic_attention_kernel(AttnArgs a) {
  extern __shared__ float qs_all[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int64_t warp = static_cast<int64_t>(blockIdx.x) * kGenericWarps + wib;
  const bool decode = a.context_lens != nullptr;
  const int n_rows = decode ? a.n_seqs : a.n_tokens;
  if (warp >= static_cast<int64_t>(n_rows) * a.n_q_heads) return;
  const int t = static_cast<int>(warp / a.n_q_heads);
  const int h = static_cast<int>(warp % a.n_q_heads);
  const int D = a.head_dim;
  const int G = a.n_q_heads / a.n_kv_heads;
  const int g = h / G;

  int s, i, limit, total;
  if (decode) {
    s = t;
    i = 0;
    total = max(a.context_lens[s], 0);
    limit = total;
  } else {
    // rows at or past the last query start are padding (a fixed-shape step
    // with fewer real tokens): no sequence owns them, their output rows stay
    // as they are, as in the tensor-core prefill
    if (t >= a.query_start_loc[a.n_seqs]) return;
    int lo = 0, hi = a.n_seqs - 1;  // last s with query_start_loc[s] <= t
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.query_start_loc[mid] <= t) lo = mid; else hi = mid - 1;
    }
    s = lo;
    i = t - a.query_start_loc[s];
    const int n_new = a.query_start_loc[s + 1] - a.query_start_loc[s];
    if (i < 0 || i >= n_new) {
      if (lane == 0) raise_flag(a.err, PKV_FLAG_BAD_QUERY_LAYOUT);
      return;
    }
    total = max(a.num_prior[s], 0) + n_new;
    limit = (n_new > 1) ? a.num_prior[s] + i + 1 : total;
  }
  const int cap = a.max_blocks * a.block_size;
  if (total > cap) {
    if (lane == 0) raise_flag(a.err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
    limit = min(limit, cap);
  }

  const T* q = static_cast<const T*>(a.q) + static_cast<int64_t>(t) * a.q_stride +
               static_cast<int64_t>(h) * D;
  float* qs = qs_all + wib * D;
  for (int d = lane; d < D; d += 32) qs[d] = Elem<T>::to_f(q[d]);
  __syncwarp();

  const int32_t* table = a.block_tables + static_cast<int64_t>(s) * a.bt_stride;

  float m = -FLT_MAX, l = 0.f;
  float acc[kGenericMaxDPerLane];
#pragma unroll
  for (int r = 0; r < kGenericMaxDPerLane; ++r) acc[r] = 0.f;
  bool bad_block = false;

  for (int j0 = 0; j0 < limit; j0 += 32) {
    const int j = j0 + lane;
    float sj = -FLT_MAX;
    if (j < limit) {
      int blk = table[j / a.block_size];
      if (blk < 0 || blk >= a.num_blocks) { bad_block = true; blk = 0; }
      const int64_t krow = (static_cast<int64_t>(blk) * a.block_size + j % a.block_size) * a.n_kv_heads + g;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(qs[d], kv_elem<T, FP8>(a.k_pool, a.k_scale, krow, D, d), dot);
      sj = dot * a.scale;
    }
    float mc = sj;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
    const float m_new = fmaxf(m, mc);
    const float corr = expf(m - m_new);
    const float pj = (j < limit) ? expf(sj - m_new) : 0.f;
    float ps = pj;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l = l * corr + ps;
#pragma unroll
    for (int r = 0; r < kGenericMaxDPerLane; ++r) acc[r] *= corr;
    const int nk = min(32, limit - j0);
    for (int jj = 0; jj < nk; ++jj) {
      const float p = __shfl_sync(0xffffffffu, pj, jj);
      const int key = j0 + jj;
      int blk = table[key / a.block_size];
      if (blk < 0 || blk >= a.num_blocks) blk = 0;
      const int64_t vrow = (static_cast<int64_t>(blk) * a.block_size + key % a.block_size) * a.n_kv_heads + g;
#pragma unroll
      for (int r = 0; r < kGenericMaxDPerLane; ++r) {
        const int d = lane + 32 * r;
        if (d < D) acc[r] = fmaf(p, kv_elem<T, FP8>(a.v_pool, a.v_scale, vrow, D, d), acc[r]);
      }
    }
    m = m_new;
  }
  if (__any_sync(0xffffffffu, bad_block) && lane == 0) raise_flag(a.err, PKV_FLAG_BLOCK_OUT_OF_RANGE);

  T* out = static_cast<T*>(a.out) + static_cast<int64_t>(t) * a.out_stride +
           static_cast<int64_t>(h) * D;
  const float inv = (limit > 0) ? 1.f / l : 0.f;
#pragma unroll
  for (int r = 0; r < kGenericMaxDPerLane; ++r) {
    const int d = lane + 32 * r;
    if (d < D) out[d] = Elem<T>::from_f(acc[r] * inv);
  }
}

cudaError_t launch_generic_attention(const AttnArgs& a, cudaStream_t stream) {
  const int n_rows = a.context_lens != nullptr ? a.n_seqs : a.n_tokens;
  const int64_t warps = static_cast<int64_t>(n_rows) * a.n_q_heads;
  if (warps == 0) return cudaSuccess;
  const int64_t grid = (warps + kGenericWarps - 1) / kGenericWarps;
  if (grid > 0x7fffffff) return cudaErrorInvalidConfiguration;
  const size_t smem = sizeof(float) * kGenericWarps * a.head_dim;
  const unsigned g = static_cast<unsigned>(grid);
  auto go = [&](auto tag, auto fp8) {
    using T = decltype(tag);
    generic_attention_kernel<T, decltype(fp8)::value><<<g, kGenericWarps * 32, smem, stream>>>(a);
  };
  const bool fp8 = a.k_scale != nullptr;
  switch (a.dtype) {
    case PKV_DTYPE_F32:
      fp8 ? go(float{}, std::true_type{}) : go(float{}, std::false_type{});
      break;
    case PKV_DTYPE_F16:
      fp8 ? go(__half{}, std::true_type{}) : go(__half{}, std::false_type{});
      break;
    default:
      fp8 ? go(__nv_bfloat16{}, std::true_type{}) : go(__nv_bfloat16{}, std::false_type{});
      break;
  }
  return cudaGetLastError();
}

}  // namespace pkv
