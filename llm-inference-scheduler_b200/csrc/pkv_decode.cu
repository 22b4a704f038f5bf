// pkv_decode.cu -- paged decode attention for B200 (sm_100a), fp16 / bf16 KV.
//
// Replaces the reference's per-sequence gather + GQA attention for one new
// token (mini_engine/paged/block_manager.py:136-141 and
// mini_engine/model/qwen2.py:98-128 with num_new == 1).
//
// Design (HBM-bound: every KV byte is read exactly once):
//  * Stream-K split.  The flattened list of all sequences' KV blocks is cut
//    into gridDim.x equal ranges, one per persistent CTA (grid = SMs x
//    resident CTAs), so lognormal context lengths cannot unbalance the GPU.
//    A CTA walks its range as segments (one per sequence it touches).
//  * Producer warp: TMA tensor loads (cp.async.bulk.tensor, 128-byte swizzle)
//    of each 16-token block, one 16x64 tile per KV head for K and for V,
//    into a kStages-deep shared-memory ring guarded by mbarriers
//    (full: transaction bytes; empty: one arrival per consumer warp).
//  * Consumer warp h (one per KV head): S = Q K^T and O += P V with the
//    m16n8k16 tensor-core MMA.  The M=16 rows are the G <= 8 query heads of
//    the GQA group, so all 7 Qwen2 query heads consume each K/V tile from one
//    shared-memory read.  Online softmax in fp32 (exp2 domain).
//  * Sequences fully inside one CTA's range are normalised and stored
//    directly.  A sequence split across CTAs leaves (m, l, O) partials in the
//    workspace; the CTA that arrives last on the sequence's counter (atomic,
//    no spinning) merges them and resets the counter to zero.
#include <float.h>

#include <mutex>
#include <unordered_map>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

constexpr int kDecStages = 6;
constexpr int kDecMaxCtas = 1024;
constexpr int kDecMaxSeqs = 2048;
constexpr int kDecMinBlocksPerCta = 4;
constexpr int kDecTile = 2048;  // 16 tokens x 64 dims x 2 bytes
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeParams {
  void* out;
  int64_t out_stride;
  const void* q;
  int64_t q_stride;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  const int32_t* context_lens;
  int n_seqs;
  int num_blocks;
  int n_q_heads;
  int n_kv_heads;
  int group;  // q heads per kv head
  float scale_log2;
  float* part_o;   // [2*kDecMaxCtas][n_q_heads][64]
  float* part_ml;  // [2*kDecMaxCtas][n_q_heads][2]
  int* counters;   // [n_seqs]
  int* err;
};

size_t decode_workspace_bytes(int n_seqs, int n_q_heads, int head_dim) {
  const size_t parts = static_cast<size_t>(2) * kDecMaxCtas * n_q_heads * (head_dim + 2) * 4;
  const size_t cnt = static_cast<size_t>(n_seqs) * 4;
  return ((parts + 255) & ~static_cast<size_t>(255)) + ((cnt + 255) & ~static_cast<size_t>(255));
}

bool decode_fast_supported(const AttnArgs& a) {
  const int G = a.n_q_heads / a.n_kv_heads;
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0; };
  return (a.dtype == PKV_DTYPE_F16 || a.dtype == PKV_DTYPE_BF16) && a.head_dim == 64 &&
         a.block_size == 16 && (a.n_kv_heads == 1 || a.n_kv_heads == 2 || a.n_kv_heads == 4) &&
         G <= 8 && a.n_seqs <= kDecMaxSeqs && (a.q_stride % 2) == 0 && (a.out_stride % 2) == 0 &&
         al(a.q, 4) && al(a.out, 4) && al(a.k_pool, 16) && al(a.v_pool, 16);
}

// exclusive scan of n values in smem (in place), result total returned to all threads
__device__ __forceinline__ int block_exclusive_scan(int* vals, int n, int* scratch) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int per = (n + nt - 1) / nt;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  int sum = 0;
  for (int i = lo; i < hi; ++i) sum += vals[i];
  // inclusive scan of per-thread sums across the block
  const int lane = tid & 31, wid = tid >> 5, nw = (nt + 31) >> 5;
  int x = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31 || tid == nt - 1) scratch[wid] = x;
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int w = 0; w < nw; ++w) { const int v = scratch[w]; scratch[w] = run; run += v; }
    scratch[nw] = run;
  }
  __syncthreads();
  int run = x - sum + scratch[wid];
  for (int i = lo; i < hi; ++i) { const int v = vals[i]; vals[i] = run; run += v; }
  const int total = scratch[nw];
  __syncthreads();
  return total;
}

// last index s in [0, n) with prefix[s] <= x (prefix non-decreasing, prefix[0] = 0)
__device__ __forceinline__ int find_seq(const int* prefix, int n, int x) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= x) lo = mid; else hi = mid - 1;
  }
  return lo;
}

template <typename T>
__device__ __forceinline__ void load_q_frag(uint32_t (&qa)[4][2], const DecodeParams& p, int s,
                                            int h, int lane) {
  const int g = lane >> 2, t = lane & 3;
  if (g < p.group) {
    const T* row = static_cast<const T*>(p.q) + static_cast<int64_t>(s) * p.q_stride +
                   static_cast<int64_t>(h * p.group + g) * 64;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      qa[kk][0] = __ldg(reinterpret_cast<const uint32_t*>(row + 16 * kk + 2 * t));
      qa[kk][1] = __ldg(reinterpret_cast<const uint32_t*>(row + 16 * kk + 8 + 2 * t));
    }
  } else {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) qa[kk][0] = qa[kk][1] = 0u;
  }
}

template <typename T>
__global__ void __launch_bounds__(160) paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                           const __grid_constant__ CUtensorMap vmap,
                                                           const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nkv = p.n_kv_heads;
  const int B = p.n_seqs;

  // ---- shared memory carve-up (tiles 1024-byte aligned for the 128B swizzle)
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const int stage_bytes = 2 * nkv * kDecTile;  // K tiles then V tiles
  uint8_t* tiles = base;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(tiles + kDecStages * stage_bytes);
  uint64_t* empty_bar = full_bar + kDecStages;
  int* misc = reinterpret_cast<int*>(empty_bar + kDecStages);  // [0]: last flag; [1..33] scan scratch
  int* prefix = misc + 40;                                     // [B+1]
  int* ctxs = prefix + (B + 1);                                // [B]

  // ---- prologue: clamp contexts, count blocks, prefix-sum them
  const int cap_tokens = p.max_blocks * 16;
  for (int s = tid; s < B; s += blockDim.x) {
    int c = p.context_lens[s];
    if (c < 0) c = 0;
    if (c > cap_tokens) {
      if (blockIdx.x == 0) raise_flag(p.err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
      c = cap_tokens;
    }
    ctxs[s] = c;
    prefix[s] = (c + 15) >> 4;
  }
  __syncthreads();
  const int total = block_exclusive_scan(prefix, B, misc + 1);
  if (tid == 0) prefix[B] = total;
  __syncthreads();

  const int per = max((total + static_cast<int>(gridDim.x) - 1) / static_cast<int>(gridDim.x),
                      kDecMinBlocksPerCta);
  const int n_active = (total + per - 1) / per;

  // zero rows for empty sequences (CTA 0 only; nobody else writes them)
  if (blockIdx.x == 0) {
    const int row = p.n_q_heads * 64;
    for (int s = 0; s < B; ++s) {
      if (prefix[s + 1] != prefix[s]) continue;
      T* o = static_cast<T*>(p.out) + static_cast<int64_t>(s) * p.out_stride;
      for (int i = tid; i < row; i += blockDim.x) o[i] = Elem<T>::from_f(0.f);
    }
  }
  if (static_cast<int>(blockIdx.x) >= n_active) return;

  const int r0 = blockIdx.x * per;
  const int r1 = min(r0 + per, total);

  if (tid == 0) {
    for (int i = 0; i < kDecStages; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], nkv);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == nkv) {
    // ======================= producer warp =======================
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    bool dead = false;
    int i = 0;
    for (int b0 = r0; b0 < r1; b0 += 32) {
      const int gb = b0 + lane;
      int id = 0;
      if (gb < r1) {
        const int s = find_seq(prefix, B, gb);
        const int jb = gb - prefix[s];
        id = __ldg(p.block_tables + static_cast<int64_t>(s) * p.bt_stride + jb);
        if (id < 0 || id >= p.num_blocks) {
          raise_flag(p.err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
          id = 0;
        }
      }
      const int n = min(32, r1 - b0);
      for (int k = 0; k < n; ++k, ++i) {
        const int blk = __shfl_sync(0xffffffffu, id, k);
        if (lane == 0 && !dead) {
          const int st = i % kDecStages;
          if (!mbar_wait(&empty_bar[st], ((i / kDecStages) & 1) ^ 1)) {
            raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
            dead = true;
          } else {
            uint8_t* stg = tiles + st * stage_bytes;
            mbar_arrive_expect_tx(&full_bar[st], stage_bytes);
            for (int hk = 0; hk < nkv; ++hk) {
              tma_load_3d(stg + hk * kDecTile, &kmap, &full_bar[st], 0, hk, blk * 16);
              tma_load_3d(stg + (nkv + hk) * kDecTile, &vmap, &full_bar[st], 0, hk, blk * 16);
            }
          }
        }
      }
    }
    return;
  }

  // ======================= consumer warps (warp = kv head) =======================
  const int h = warp;
  const int g = lane >> 2, t = lane & 3;
  const bool row_ok = g < p.group;
  const int qh = h * p.group + g;
  const int cons_threads = nkv * 32;
  bool dead = false;

  int s = find_seq(prefix, B, r0);
  uint32_t qa[4][2];
  load_q_frag<T>(qa, p, s, h, lane);
  int pos = r0;
  int i = 0;
  while (pos < r1) {
    const int seg_end = min(prefix[s + 1], r1);
    const int jb0 = pos - prefix[s];
    const bool complete = prefix[s] >= r0 && prefix[s + 1] <= r1;
    int s_next = s + 1;
    while (s_next < B && prefix[s_next + 1] == prefix[s_next]) ++s_next;
    uint32_t qn[4][2];
    if (seg_end < r1) load_q_frag<T>(qn, p, s_next, h, lane);

    const int ctx = ctxs[s];
    float m = -INFINITY, l = 0.f;
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    for (int jb = jb0; jb < jb0 + (seg_end - pos); ++jb, ++i) {
      const int st = i % kDecStages;
      if (!dead && !mbar_wait(&full_bar[st], (i / kDecStages) & 1)) {
        if (lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
        dead = true;
      }
      const uint32_t kt = smem_u32(tiles + st * stage_bytes + h * kDecTile);
      const uint32_t vt = smem_u32(tiles + st * stage_bytes + (nkv + h) * kDecTile);
      // ---- S = Q K^T : rows = query heads of the group, cols = 16 tokens
      float sc[2][4];
#pragma unroll
      for (int n = 0; n < 2; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int row = (lane & 7) + ((lane >> 4) << 3);
        const int chunk = 2 * kk + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kt + row * 128 + ((chunk ^ (row & 7)) << 4), b0, b1, b2, b3);
        const uint32_t a[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
        mma16816<T>(sc[0], a, b0, b1);
        mma16816<T>(sc[1], a, b2, b3);
      }
      // ---- online softmax (exp2 domain), tokens >= valid are masked
      const int valid = min(16, ctx - jb * 16);
      float x[4] = {sc[0][0] * p.scale_log2, sc[0][1] * p.scale_log2, sc[1][0] * p.scale_log2,
                    sc[1][1] * p.scale_log2};
      if (2 * t >= valid) x[0] = -INFINITY;
      if (2 * t + 1 >= valid) x[1] = -INFINITY;
      if (8 + 2 * t >= valid) x[2] = -INFINITY;
      if (9 + 2 * t >= valid) x[3] = -INFINITY;
      float mloc = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
      mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 1));
      mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 2));
      const float m_new = fmaxf(m, mloc);
      const float corr = exp2f(m - m_new);
      const float p0 = exp2f(x[0] - m_new), p1 = exp2f(x[1] - m_new);
      const float p2 = exp2f(x[2] - m_new), p3 = exp2f(x[3] - m_new);
      l = l * corr + (p0 + p1) + (p2 + p3);
      m = m_new;
#pragma unroll
      for (int j = 0; j < 8; ++j) { o[j][0] *= corr; o[j][1] *= corr; }
      // ---- O += P V : P (rows = heads, k = 16 tokens) straight from the S fragments
      const uint32_t pa[4] = {pack2<T>(p0, p1), 0u, pack2<T>(p2, p3), 0u};
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int mi = lane >> 3;
        const int row = (lane & 7) + ((mi & 1) << 3);
        const int chunk = 2 * jj + (mi >> 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vt + row * 128 + ((chunk ^ (row & 7)) << 4), v0, v1, v2, v3);
        mma16816<T>(o[2 * jj], pa, v0, v1);
        mma16816<T>(o[2 * jj + 1], pa, v2, v3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[st]);
    }

    // ---- segment epilogue
    float lt = l + __shfl_xor_sync(0xffffffffu, l, 1);
    lt += __shfl_xor_sync(0xffffffffu, lt, 2);
    if (complete) {
      if (row_ok) {
        const float inv = 1.f / lt;
        T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(s) * p.out_stride +
                  static_cast<int64_t>(qh) * 64;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<uint32_t*>(orow + 8 * j + 2 * t) = pack2<T>(o[j][0] * inv, o[j][1] * inv);
      }
    } else {
      const int slot = (prefix[s] <= r0) ? 2 * blockIdx.x : 2 * blockIdx.x + 1;
      if (row_ok) {
        float* po = p.part_o + (static_cast<int64_t>(slot) * p.n_q_heads + qh) * 64;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float2*>(po + 8 * j + 2 * t) = make_float2(o[j][0], o[j][1]);
        if (t == 0) {
          float* pml = p.part_ml + (static_cast<int64_t>(slot) * p.n_q_heads + qh) * 2;
          pml[0] = m;
          pml[1] = lt;
        }
      }
      __threadfence();
      named_bar_sync(1, cons_threads);
      if (tid == 0) {
        const int c_first = prefix[s] / per, c_last = (prefix[s + 1] - 1) / per;
        const int old = atomicAdd(p.counters + s, 1);
        const int last = (old == c_last - c_first) ? 1 : 0;
        if (last) p.counters[s] = 0;
        misc[0] = last;
      }
      named_bar_sync(1, cons_threads);
      if (misc[0]) {
        __threadfence();
        const int c_first = prefix[s] / per, c_last = (prefix[s + 1] - 1) / per;
        const int n_out = p.n_q_heads * 64;
        for (int idx = tid; idx < n_out; idx += cons_threads) {
          const int hh = idx >> 6;
          float M = -INFINITY;
          for (int c = c_first; c <= c_last; ++c) {
            const int sl = (c == c_first && prefix[s] > c * per) ? 2 * c + 1 : 2 * c;
            M = fmaxf(M, __ldcg(p.part_ml + (static_cast<int64_t>(sl) * p.n_q_heads + hh) * 2));
          }
          float L = 0.f, acc = 0.f;
          for (int c = c_first; c <= c_last; ++c) {
            const int sl = (c == c_first && prefix[s] > c * per) ? 2 * c + 1 : 2 * c;
            const float* pml = p.part_ml + (static_cast<int64_t>(sl) * p.n_q_heads + hh) * 2;
            const float w = exp2f(__ldcg(pml) - M);
            L += w * __ldcg(pml + 1);
            acc += w * __ldcg(p.part_o + static_cast<int64_t>(sl) * p.n_q_heads * 64 + idx);
          }
          T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(s) * p.out_stride;
          orow[idx] = Elem<T>::from_f(acc / L);
        }
      }
    }
    pos = seg_end;
    s = s_next;
    if (pos < r1) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) { qa[kk][0] = qn[kk][0]; qa[kk][1] = qn[kk][1]; }
    }
  }
}

size_t decode_smem_bytes(int nkv, int n_seqs) {
  return 1024 + static_cast<size_t>(kDecStages) * 2 * nkv * kDecTile +
         2 * kDecStages * sizeof(uint64_t) + 40 * sizeof(int) +
         (2 * static_cast<size_t>(n_seqs) + 1) * sizeof(int);
}

namespace {
struct OccKey {
  int dev, dtype, smem, threads;
  bool operator==(const OccKey& o) const {
    return dev == o.dev && dtype == o.dtype && smem == o.smem && threads == o.threads;
  }
};
struct OccHash {
  size_t operator()(const OccKey& k) const {
    return (static_cast<size_t>(k.dev) * 131 + k.dtype) * 1000003u + k.smem * 7 + k.threads;
  }
};
std::mutex g_occ_mu;
std::unordered_map<OccKey, int, OccHash> g_occ;
}  // namespace

cudaError_t launch_decode_fast(const AttnArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap,
                               void* workspace, cudaStream_t stream) {
  if (a.n_seqs == 0) return cudaSuccess;
  const int nkv = a.n_kv_heads;
  const int threads = 32 * (nkv + 1);
  const size_t smem = decode_smem_bytes(nkv, a.n_seqs);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  auto kern = a.dtype == PKV_DTYPE_F16 ? paged_decode_kernel<__half> : paged_decode_kernel<__nv_bfloat16>;
  int grid = 0;
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    const OccKey key{dev, a.dtype, static_cast<int>(smem), threads};
    auto it = g_occ.find(key);
    if (it == g_occ.end()) {
      // one opt-in size per (device, kernel): the largest any call can need
      const OccKey attr_key{dev, a.dtype, -1, 0};
      if (g_occ.find(attr_key) == g_occ.end()) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(decode_smem_bytes(4, kDecMaxSeqs)));
        if (e != cudaSuccess) return e;
        g_occ.emplace(attr_key, 0);
      }
      int per_sm = 0, sms = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      it = g_occ.emplace(key, std::max(1, std::min(kDecMaxCtas, per_sm * sms))).first;
    }
    grid = it->second;
  }
  DecodeParams p;
  p.out = a.out;
  p.out_stride = a.out_stride;
  p.q = a.q;
  p.q_stride = a.q_stride;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.max_blocks = a.max_blocks;
  p.context_lens = a.context_lens;
  p.n_seqs = a.n_seqs;
  p.num_blocks = a.num_blocks;
  p.n_q_heads = a.n_q_heads;
  p.n_kv_heads = nkv;
  p.group = a.n_q_heads / nkv;
  p.scale_log2 = a.scale * kLog2e;
  const size_t parts_o = static_cast<size_t>(2) * kDecMaxCtas * a.n_q_heads * 64 * 4;
  const size_t parts_ml = static_cast<size_t>(2) * kDecMaxCtas * a.n_q_heads * 2 * 4;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float*>(ws + parts_o);
  p.counters = reinterpret_cast<int*>(ws + ((parts_o + parts_ml + 255) & ~static_cast<size_t>(255)));
  p.err = a.err;
  kern<<<grid, threads, smem, stream>>>(*kmap, *vmap, p);
  return cudaGetLastError();
}

}  // namespace pkv
