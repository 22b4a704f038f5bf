// pkv_rope.cu -- rotary embedding of q and k fused with the KV append.
//
// Replaces, per layer, the reference's RoPE of the projected q and k
// (mini_engine/model/qwen2.py:152-158: K is stored post-RoPE) followed by the
// scatter of k and v into the block pool (PagedKVCache.append_and_fetch,
// mini_engine/paged/block_manager.py:121-131).  Input is the fused q|k|v
// projection row of each token; output is the rotated q (for the attention
// kernels) and the rotated k plus v written at the token's slot.
//
// Rotation (half-split pairs, as the reference and Hugging Face Qwen2):
//   out[i]        = x[i] * cos[p, i]        - x[i + D/2] * sin[p, i]
//   out[i + D/2]  = x[i + D/2] * cos[p, i + D/2] + x[i] * sin[p, i + D/2]
// with the model's own cos/sin tables (computed in fp32, stored in the model
// dtype).  Each product and the sum are rounded to the element type exactly
// as the separate elementwise operations of the unfused path round them
// (multiply in fp32, round; add in fp32, round; no fused multiply-add), so
// the result is bit-identical to that path for fp32, fp16 and bf16.
//
// Two forms.  Where each half of a head row is a whole number of 16-byte
// vectors at aligned addresses (head_dim 64 in fp16 / bf16 / fp32), a head
// is served by D / (2 V) threads that each move one vector of each half with
// 16-byte loads and stores (rope_reshape_and_cache_vec_kernel).  Otherwise
// one warp per (token, head) of the projection row (Hq query heads, Hkv key
// heads, Hkv value heads): lane l owns the pairs (i, i + D/2) for i = l,
// l + 32, ...  Both give every (token, head) its own threads, so a decode step
// of B tokens spreads over B x (Hq + 2 Hkv) heads' worth of independent work
// (one warp per token looping over the heads left a 64-token step
// latency-bound on 8 SMs).
#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

template <typename E> __device__ __forceinline__ E rnd(float x);
template <> __device__ __forceinline__ float rnd<float>(float x) { return x; }
template <> __device__ __forceinline__ __half rnd<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 rnd<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <typename E> __device__ __forceinline__ float tof(E x) { return static_cast<float>(x); }
template <> __device__ __forceinline__ float tof<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float tof<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

// a * c + b * s with the unfused path's rounding: each product rounded to E,
// then the sum rounded to E
template <typename E>
__device__ __forceinline__ E rot_term(float a, float c, float b, float s) {
  const float p = tof<E>(rnd<E>(__fmul_rn(a, c)));
  const float q = tof<E>(rnd<E>(__fmul_rn(b, s)));
  return rnd<E>(__fadd_rn(p, q));
}

template <typename E>
__global__ void __launch_bounds__(256) rope_reshape_and_cache_kernel(
    E* __restrict__ q_out, int64_t q_out_stride, const E* __restrict__ qkv, int64_t qkv_stride,
    const int64_t* __restrict__ positions, const E* __restrict__ cos_t,
    const E* __restrict__ sin_t, int64_t max_pos, E* __restrict__ k_pool, E* __restrict__ v_pool,
    const int64_t* __restrict__ slots, int64_t n_slots, int n_tokens, int hq, int hkv, int d,
    int* err) {
  // launched with programmatic serialization: wait for the preceding grid
  // (it may still read the pool or write qkv), then let the next kernel's
  // prologue start
  pdl_wait();
  pdl_trigger();
  const int heads = hq + 2 * hkv;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(n_tokens) * heads) return;
  const int t = static_cast<int>(w / heads);
  const int h = static_cast<int>(w - static_cast<int64_t>(t) * heads);
  const int64_t pos = __ldg(positions + t);
  if (pos < 0 || pos >= max_pos) {
    if (lane == 0 && h == 0) raise_flag(err, PKV_FLAG_POSITION_OUT_OF_RANGE);
    return;
  }
  const int64_t slot = __ldg(slots + t);
  if (slot >= n_slots && lane == 0 && h == 0) raise_flag(err, PKV_FLAG_SLOT_OUT_OF_RANGE);
  const bool store_kv = slot >= 0 && slot < n_slots;  // slot -1: padding token
  if (h >= hq && !store_kv) return;
  const E* x = qkv + static_cast<int64_t>(t) * qkv_stride + static_cast<int64_t>(h) * d;
  if (h >= hq + hkv) {  // v: as projected
    E* vdst = v_pool + slot * (static_cast<int64_t>(hkv) * d) + static_cast<int64_t>(h - hq - hkv) * d;
    for (int i = lane; i < d; i += 32) vdst[i] = __ldg(x + i);
    return;
  }
  const E* cr = cos_t + pos * d;
  const E* sr = sin_t + pos * d;
  const int half = d >> 1;
  E* dst = h < hq ? q_out + static_cast<int64_t>(t) * q_out_stride + static_cast<int64_t>(h) * d
                  : k_pool + slot * (static_cast<int64_t>(hkv) * d) + static_cast<int64_t>(h - hq) * d;
  for (int i = lane; i < half; i += 32) {
    const float c1 = tof<E>(__ldg(cr + i)), c2 = tof<E>(__ldg(cr + i + half));
    const float s1 = tof<E>(__ldg(sr + i)), s2 = tof<E>(__ldg(sr + i + half));
    const float x1 = tof<E>(__ldg(x + i)), x2 = tof<E>(__ldg(x + i + half));
    dst[i] = rot_term<E>(x1, c1, -x2, s1);
    dst[i + half] = rot_term<E>(x2, c2, x1, s2);
  }
}

// fp8 e4m3 pools: the same rotation, then the rotated k and the v rows are
// quantised per (token, KV head) exactly as reshape_and_cache_fp8 quantises
// its input (scale = absmax / 448, value = e4m3(x / scale), RNE, saturated):
// bit-identical to rotating in the model dtype and calling that append.  A
// head's values are produced twice by each lane (once for the warp absmax,
// once to quantise), so any head_dim works.
template <typename E>
__global__ void __launch_bounds__(256) rope_reshape_and_cache_fp8_kernel(
    E* __restrict__ q_out, int64_t q_out_stride, const E* __restrict__ qkv, int64_t qkv_stride,
    const int64_t* __restrict__ positions, const E* __restrict__ cos_t,
    const E* __restrict__ sin_t, int64_t max_pos, uint8_t* __restrict__ k_pool,
    uint8_t* __restrict__ v_pool, float* __restrict__ k_scale, float* __restrict__ v_scale,
    const int64_t* __restrict__ slots, int64_t n_slots, int n_tokens, int hq, int hkv, int d,
    int* err) {
  pdl_wait();
  pdl_trigger();
  const int heads = hq + 2 * hkv;
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(n_tokens) * heads) return;  // warp-uniform
  const int t = static_cast<int>(w / heads);
  const int h = static_cast<int>(w - static_cast<int64_t>(t) * heads);
  const int64_t pos = __ldg(positions + t);
  if (pos < 0 || pos >= max_pos) {
    if (lane == 0 && h == 0) raise_flag(err, PKV_FLAG_POSITION_OUT_OF_RANGE);
    return;
  }
  const int64_t slot = __ldg(slots + t);
  if (slot >= n_slots && lane == 0 && h == 0) raise_flag(err, PKV_FLAG_SLOT_OUT_OF_RANGE);
  const bool store_kv = slot >= 0 && slot < n_slots;  // slot -1: padding token
  if (h >= hq && !store_kv) return;
  const E* x = qkv + static_cast<int64_t>(t) * qkv_stride + static_cast<int64_t>(h) * d;
  const E* cr = cos_t + pos * d;
  const E* sr = sin_t + pos * d;
  const int half = d >> 1;
  // rotated element pair (i, i + half) of this head
  auto rot = [&](int i, E& o1, E& o2) {
    const float c1 = tof<E>(__ldg(cr + i)), c2 = tof<E>(__ldg(cr + i + half));
    const float s1 = tof<E>(__ldg(sr + i)), s2 = tof<E>(__ldg(sr + i + half));
    const float x1 = tof<E>(__ldg(x + i)), x2 = tof<E>(__ldg(x + i + half));
    o1 = rot_term<E>(x1, c1, -x2, s1);
    o2 = rot_term<E>(x2, c2, x1, s2);
  };
  if (h < hq) {
    E* qrow = q_out + static_cast<int64_t>(t) * q_out_stride + static_cast<int64_t>(h) * d;
    for (int i = lane; i < half; i += 32) {
      E o1, o2;
      rot(i, o1, o2);
      qrow[i] = o1;
      qrow[i + half] = o2;
    }
    return;
  }
  float amax = 0.f;
  if (h < hq + hkv) {  // k: rotated
    const int kh = h - hq;
    for (int i = lane; i < half; i += 32) {
      E o1, o2;
      rot(i, o1, o2);
      amax = fmaxf(amax, fmaxf(fabsf(tof<E>(o1)), fabsf(tof<E>(o2))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = fp8_row_scale(amax);
    uint8_t* kd = k_pool + (slot * hkv + kh) * d;
    for (int i = lane; i < half; i += 32) {
      E o1, o2;
      rot(i, o1, o2);
      kd[i] = fp8_quantize(tof<E>(o1), sc);
      kd[i + half] = fp8_quantize(tof<E>(o2), sc);
    }
    if (lane == 0) k_scale[slot * hkv + kh] = sc;
    return;
  }
  const int vh = h - hq - hkv;  // v: as projected
  for (int i = lane; i < d; i += 32) amax = fmaxf(amax, fabsf(tof<E>(__ldg(x + i))));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float sc = fp8_row_scale(amax);
  uint8_t* vd = v_pool + (slot * hkv + vh) * d;
  for (int i = lane; i < d; i += 32) vd[i] = fp8_quantize(tof<E>(__ldg(x + i)), sc);
  if (lane == 0) v_scale[slot * hkv + vh] = sc;
}

// The same rotation and append over 16-byte vectors, for rows whose halves
// are whole vectors (D/2 x sizeof(E) a multiple of 16) at 16-byte aligned
// addresses.  A head of D values is served by TH = D / (2 V) threads (V =
// 16 / sizeof(E) values a vector): thread j loads vector j of the first half
// and its partner vector j of the second half, with the matching cos / sin
// vectors, so every load and store is a full 16-byte access and a warp
// covers 32 / TH heads of a token row.  Element by element the arithmetic is
// rot_term's, so the outputs equal the warp-per-head kernels' bit for bit.
// FP8: the head's absmax is reduced over its TH lanes (an aligned group of
// the warp; every control-flow decision above the reduction is uniform over
// the group) and each lane writes its 2 x V bytes.
template <typename E, bool FP8>
__global__ void __launch_bounds__(256) rope_reshape_and_cache_vec_kernel(
    E* __restrict__ q_out, int64_t q_out_stride, const E* __restrict__ qkv, int64_t qkv_stride,
    const int64_t* __restrict__ positions, const E* __restrict__ cos_t,
    const E* __restrict__ sin_t, int64_t max_pos, void* __restrict__ k_pool,
    void* __restrict__ v_pool, float* __restrict__ k_scale, float* __restrict__ v_scale,
    const int64_t* __restrict__ slots, int64_t n_slots, int n_tokens, int hq, int hkv, int d,
    int* err) {
  constexpr int V = 16 / sizeof(E);
  union Vec {
    uint4 u;
    E e[V];
  };
  pdl_wait();
  pdl_trigger();
  const int th = d / (2 * V);
  const int heads = hq + 2 * hkv;
  const int64_t per_tok = static_cast<int64_t>(heads) * th;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= per_tok * n_tokens) return;  // uniform over each group of th lanes
  const int t = static_cast<int>(g / per_tok);
  const int r = static_cast<int>(g - t * per_tok);
  const int h = r / th;
  const int j = r - h * th;
  const int64_t pos = __ldg(positions + t);
  if (pos < 0 || pos >= max_pos) {
    if (r == 0) raise_flag(err, PKV_FLAG_POSITION_OUT_OF_RANGE);
    return;
  }
  const int64_t slot = __ldg(slots + t);
  if (slot >= n_slots && r == 0) raise_flag(err, PKV_FLAG_SLOT_OUT_OF_RANGE);
  const bool store_kv = slot >= 0 && slot < n_slots;  // slot -1: padding token
  if (h >= hq && !store_kv) return;
  const int half = d >> 1;
  const E* x = qkv + static_cast<int64_t>(t) * qkv_stride + static_cast<int64_t>(h) * d + j * V;
  Vec a, b;  // values [jV, jV + V) and [half + jV, half + jV + V) of the head
  a.u = __ldg(reinterpret_cast<const uint4*>(x));
  b.u = __ldg(reinterpret_cast<const uint4*>(x + half));
  const int lane = threadIdx.x & 31;
  const unsigned group = th >= 32 ? 0xffffffffu : ((1u << th) - 1u) << (lane & ~(th - 1));
  // FP8: this head's row (KV head kh of the slot) quantised from a and b
  auto store_fp8 = [&](uint8_t* pool, float* scales, int kh) {
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < V; ++k)
      amax = fmaxf(amax, fmaxf(fabsf(tof<E>(a.e[k])), fabsf(tof<E>(b.e[k]))));
    for (int o = th >> 1; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(group, amax, o));
    const float sc = fp8_row_scale(amax);
    uint32_t qa[V / 2], qb[V / 2];
#pragma unroll
    for (int k = 0; k < V / 2; ++k) {
      qa[k] = e4m3x2_rn_sat(__fdiv_rn(tof<E>(a.e[2 * k]), sc), __fdiv_rn(tof<E>(a.e[2 * k + 1]), sc));
      qb[k] = e4m3x2_rn_sat(__fdiv_rn(tof<E>(b.e[2 * k]), sc), __fdiv_rn(tof<E>(b.e[2 * k + 1]), sc));
    }
    uint8_t* row = pool + (slot * hkv + kh) * d;
    if constexpr (V == 8) {  // 8 bytes a half-vector
      *reinterpret_cast<uint2*>(row + j * V) = make_uint2(qa[0] | (qa[1] << 16), qa[2] | (qa[3] << 16));
      *reinterpret_cast<uint2*>(row + half + j * V) =
          make_uint2(qb[0] | (qb[1] << 16), qb[2] | (qb[3] << 16));
    } else {  // V == 4: 4 bytes
      *reinterpret_cast<uint32_t*>(row + j * V) = qa[0] | (qa[1] << 16);
      *reinterpret_cast<uint32_t*>(row + half + j * V) = qb[0] | (qb[1] << 16);
    }
    if (j == 0) scales[slot * hkv + kh] = sc;
  };
  if (h >= hq + hkv) {  // v: as projected
    const int vh = h - hq - hkv;
    if constexpr (FP8) {
      store_fp8(static_cast<uint8_t*>(v_pool), v_scale, vh);
    } else {
      E* vd = static_cast<E*>(v_pool) + (slot * hkv + vh) * d + j * V;
      *reinterpret_cast<uint4*>(vd) = a.u;
      *reinterpret_cast<uint4*>(vd + half) = b.u;
    }
    return;
  }
  Vec c1, c2, s1, s2;
  const E* cr = cos_t + pos * d + j * V;
  const E* sr = sin_t + pos * d + j * V;
  c1.u = __ldg(reinterpret_cast<const uint4*>(cr));
  c2.u = __ldg(reinterpret_cast<const uint4*>(cr + half));
  s1.u = __ldg(reinterpret_cast<const uint4*>(sr));
  s2.u = __ldg(reinterpret_cast<const uint4*>(sr + half));
  Vec o1, o2;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const float x1 = tof<E>(a.e[k]), x2 = tof<E>(b.e[k]);
    o1.e[k] = rot_term<E>(x1, tof<E>(c1.e[k]), -x2, tof<E>(s1.e[k]));
    o2.e[k] = rot_term<E>(x2, tof<E>(c2.e[k]), x1, tof<E>(s2.e[k]));
  }
  if (h < hq) {
    E* qd = q_out + static_cast<int64_t>(t) * q_out_stride + static_cast<int64_t>(h) * d + j * V;
    *reinterpret_cast<uint4*>(qd) = o1.u;
    *reinterpret_cast<uint4*>(qd + half) = o2.u;
    return;
  }
  const int kh = h - hq;  // k: rotated
  if constexpr (FP8) {
    a = o1;
    b = o2;
    store_fp8(static_cast<uint8_t*>(k_pool), k_scale, kh);
  } else {
    E* kd = static_cast<E*>(k_pool) + (slot * hkv + kh) * d + j * V;
    *reinterpret_cast<uint4*>(kd) = o1.u;
    *reinterpret_cast<uint4*>(kd + half) = o2.u;
  }
}

// the vectorised kernel applies: halves of whole 16-byte vectors, at most
// 32 threads a head, every row start 16-byte aligned
static bool rope_vec_ok(const RopeArgs& a, int esize) {
  const int v = 16 / esize;
  if (a.head_dim % (2 * v) != 0) return false;
  const int th = a.head_dim / (2 * v);
  if (th > 32 || (th & (th - 1)) != 0) return false;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a.q_out) || !al(a.qkv) || !al(a.cos_t) || !al(a.sin_t) || !al(a.k_pool) || !al(a.v_pool))
    return false;
  return (a.q_out_stride * esize) % 16 == 0 && (a.qkv_stride * esize) % 16 == 0;
}

cudaError_t launch_rope_reshape_and_cache(const RopeArgs& a, cudaStream_t stream) {
  if (a.n_tokens == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t warps = static_cast<int64_t>(a.n_tokens) * (a.n_q_heads + 2 * a.n_kv_heads);
  if ((warps + 7) / 8 > 0x7fffffff) return cudaErrorInvalidValue;
  const int grid = static_cast<int>((warps + 7) / 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int64_t n_slots = static_cast<int64_t>(a.num_blocks) * a.block_size;
  auto go = [&](auto tag) {
    using E = decltype(tag);
    if (rope_vec_ok(a, sizeof(E))) {
      const int64_t th = a.head_dim / (2 * (16 / static_cast<int>(sizeof(E))));
      const int64_t n = static_cast<int64_t>(a.n_tokens) * (a.n_q_heads + 2 * a.n_kv_heads) * th;
      if ((n + threads - 1) / threads > 0x7fffffff) return cudaErrorInvalidValue;
      cfg.gridDim = dim3(static_cast<unsigned>((n + threads - 1) / threads));
      auto kern = a.k_scale != nullptr ? rope_reshape_and_cache_vec_kernel<E, true>
                                       : rope_reshape_and_cache_vec_kernel<E, false>;
      return cudaLaunchKernelEx(&cfg, kern, static_cast<E*>(a.q_out), a.q_out_stride,
                                static_cast<const E*>(a.qkv), a.qkv_stride, a.positions,
                                static_cast<const E*>(a.cos_t), static_cast<const E*>(a.sin_t),
                                static_cast<int64_t>(a.max_pos), a.k_pool, a.v_pool, a.k_scale,
                                a.v_scale, a.slots, n_slots, a.n_tokens, a.n_q_heads, a.n_kv_heads,
                                a.head_dim, a.err);
    }
    if (a.k_scale != nullptr)
      return cudaLaunchKernelEx(&cfg, rope_reshape_and_cache_fp8_kernel<E>, static_cast<E*>(a.q_out),
                                a.q_out_stride, static_cast<const E*>(a.qkv), a.qkv_stride,
                                a.positions, static_cast<const E*>(a.cos_t),
                                static_cast<const E*>(a.sin_t), static_cast<int64_t>(a.max_pos),
                                static_cast<uint8_t*>(a.k_pool), static_cast<uint8_t*>(a.v_pool),
                                a.k_scale, a.v_scale, a.slots, n_slots, a.n_tokens, a.n_q_heads,
                                a.n_kv_heads, a.head_dim, a.err);
    return cudaLaunchKernelEx(&cfg, rope_reshape_and_cache_kernel<E>, static_cast<E*>(a.q_out),
                              a.q_out_stride, static_cast<const E*>(a.qkv), a.qkv_stride,
                              a.positions, static_cast<const E*>(a.cos_t),
                              static_cast<const E*>(a.sin_t), static_cast<int64_t>(a.max_pos),
                              static_cast<E*>(a.k_pool), static_cast<E*>(a.v_pool), a.slots, n_slots,
                              a.n_tokens, a.n_q_heads, a.n_kv_heads, a.head_dim, a.err);
  };
  if (a.dtype == PKV_DTYPE_F32) return go(float{});
  if (a.dtype == PKV_DTYPE_F16) return go(__half{});
  return go(__nv_bfloat16{});
}

}  // namespace pkv
