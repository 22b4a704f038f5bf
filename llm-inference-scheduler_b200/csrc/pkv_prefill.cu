// pkv_prefill.cu -- paged chunked-prefill attention on the 5th-generation tensor
// cores (tcgen05 + tensor memory), fp16 / bf16 KV, head_dim 64, 16-token blocks.
//
// Replaces the reference's per-sequence gather + _attention for num_new > 1
// (mini_engine/paged/block_manager.py:136-141, mini_engine/model/qwen2.py:98-128):
// query i of sequence s attends to keys 0 .. num_prior[s] + i, with the prefix
// blocks (shared radix-cache blocks included) read in place through the
// block table.
//
// One CTA per (sequence, query head, tile of 128 queries); 6 warps:
//  * warps 0-3 (softmax): thread r owns query row r.  It reads its row of
//    S = Q K^T from TMEM (tcgen05.ld), applies the scale, the causal mask and
//    an online softmax in the exp2 domain, writes P (fp16/bf16) into a
//    128-byte-swizzled shared tile, and at the end reads O from TMEM,
//    normalises and stores it.  O is rescaled in TMEM only when the running
//    maximum grows by more than 8 (2^8 bounds P), so rescaling is rare.
//  * warp 4 (producer): TMA tensor loads of the Q tile (once) and, per key
//    tile of 128 keys (8 blocks), the K and V blocks into a 3-stage ring;
//    blocks past the visible keys are fetched from an out-of-range coordinate
//    and arrive as zeros.
//  * warp 5 (MMA): allocates 512 TMEM columns (S double buffer 2 x 128,
//    O 64) and one thread issues tcgen05.mma kind::f16 (M=128):
//    S_j = Q K_j^T (N=128, K=64, both K-major), O += P_j V_j (N=64, K=128;
//    V is the MN-major B operand), committing to mbarriers.  S_{j+1} is issued
//    before waiting for P_j, so QK^T overlaps the softmax.
// Every wait is bounded; on a timeout the kernel flags PKV_FLAG_PIPELINE_TIMEOUT,
// stops waiting and still frees its tensor memory.
#include <float.h>

#include <mutex>
#include <type_traits>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

constexpr int kPfM = 128;                 // query rows per CTA
constexpr int kPfN = 128;                 // keys per tile (8 blocks of 16)
constexpr int kPfStages = 3;              // K/V ring depth
constexpr int kPfTile = 128 * 64 * 2;     // 16 KB: 128 rows x 64 dims x 2 bytes
constexpr int kPfThreads = 192;
constexpr uint32_t kPfTmemCols = 512;

// shared-memory offsets from the 1024-byte aligned base
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kPfTile;
constexpr int kOffV = kOffK + kPfStages * kPfTile;
constexpr int kOffP = kOffV + kPfStages * kPfTile;   // 2 buffers x (2 sub-tiles x 16 KB)
constexpr int kOffBar = kOffP + 2 * 2 * kPfTile;
constexpr int kNumBars = 1 + 2 * kPfStages + 2 + 2 + 2 + 2;
constexpr int kPfSmemBytes = 1024 + kOffBar + kNumBars * 8 + 16;

struct PrefillParams {
  void* out;
  int64_t out_stride;
  const int32_t* block_tables;
  int64_t bt_stride;
  int max_blocks;
  const int32_t* qsl;
  const int32_t* num_prior;
  int num_blocks;
  int n_tokens;
  int group;
  float scale_log2;
  int* err;
};

template <typename T>
__global__ void __launch_bounds__(kPfThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int qt = blockIdx.x, h = blockIdx.y, s = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int q_begin = p.qsl[s];
  const int n_new = p.qsl[s + 1] - q_begin;
  const int q0 = qt * kPfM;
  if (qt == static_cast<int>(gridDim.x) - 1 && n_new > static_cast<int>(gridDim.x) * kPfM && tid == 0)
    raise_flag(p.err, PKV_FLAG_BAD_QUERY_LAYOUT);  // max_query_len below a chunk length
  if (q_begin < 0 || n_new < 0 || q_begin + n_new > p.n_tokens) {
    if (qt == 0 && h == 0 && tid == 0) raise_flag(p.err, PKV_FLAG_BAD_QUERY_LAYOUT);
    return;
  }
  if (n_new == 0 || q0 >= n_new) return;  // uniform: before any barrier or allocation
  const int prior = max(p.num_prior[s], 0);
  const int rows = min(kPfM, n_new - q0);
  int kv_len = prior + q0 + rows;  // keys visible to this tile's last row
  const int cap = p.max_blocks * 16;
  if (kv_len > cap) {
    if (tid == 0) raise_flag(p.err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
    kv_len = cap;
  }
  const int n_tiles = (kv_len + kPfN - 1) / kPfN;
  const int nb_needed = (kv_len + 15) >> 4;
  const int g = h / p.group;

  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kPfStages;
  uint64_t* s_full = kv_empty + kPfStages;
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* o_done = p_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const uint32_t sbase = smem_u32(base);

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kPfStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, kPfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t t_o = tbase + 256;

  if (warp == 4) {
    // ======================= producer =======================
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_arrive_expect_tx(q_full, kPfTile);
      tma_load_3d(base + kOffQ, &qmap, q_full, 0, h, q_begin + q0);
    }
    bool dead = false;
    for (int j = 0; j < n_tiles; ++j) {
      int tok = p.num_blocks * 16;  // out of range: TMA fills zeros
      if (lane < 8) {
        const int jb = j * 8 + lane;
        if (jb < nb_needed) {
          int id = __ldg(p.block_tables + static_cast<int64_t>(s) * p.bt_stride + jb);
          if (id < 0 || id >= p.num_blocks) {
            raise_flag(p.err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
            id = 0;
          }
          tok = id * 16;
        }
      }
      int toks[8];
#pragma unroll
      for (int b = 0; b < 8; ++b) toks[b] = __shfl_sync(0xffffffffu, tok, b);
      if (lane == 0 && !dead) {
        const int st = j % kPfStages;
        if (!mbar_wait(&kv_empty[st], ((j / kPfStages) & 1) ^ 1)) {
          raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
          dead = true;
        } else {
          mbar_arrive_expect_tx(&kv_full[st], 2 * kPfTile);
          uint8_t* kd = base + kOffK + st * kPfTile;
          uint8_t* vd = base + kOffV + st * kPfTile;
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            tma_load_3d(kd + b * 2048, &kmap, &kv_full[st], 0, g, toks[b]);
            tma_load_3d(vd + b * 2048, &vmap, &kv_full[st], 0, g, toks[b]);
          }
        }
      }
    }
  } else if (warp == 5) {
    // ======================= MMA issuer (one thread) =======================
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc_s = mma_idesc_f16(fmt, 0, 0, kPfN, kPfM);
      constexpr uint32_t idesc_o = mma_idesc_f16(fmt, 0, 1, 64, kPfM);
      bool dead = !mbar_wait(q_full, 0);
      auto issue_qk = [&](int j) {
        const int st = j % kPfStages, sb = j & 1;
        if (!dead && !mbar_wait(&kv_full[st], (j / kPfStages) & 1)) dead = true;
        if (!dead && !mbar_wait(&s_empty[sb], ((j >> 1) & 1) ^ 1)) dead = true;
        if (dead) return;
        tc_fence_after();
        const uint32_t qa = sbase + kOffQ, ka = sbase + kOffK + st * kPfTile;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(tbase + sb * 128, smem_desc(qa + kk * 32, 16, 1024),
                     smem_desc(ka + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[sb]);
      };
      issue_qk(0);
      for (int j = 0; j < n_tiles; ++j) {
        if (j + 1 < n_tiles) issue_qk(j + 1);
        const int st = j % kPfStages, pb = j & 1;
        if (!dead && !mbar_wait(&p_full[pb], (j >> 1) & 1)) dead = true;
        if (dead) break;
        tc_fence_after();
        const uint32_t pa = sbase + kOffP + pb * 2 * kPfTile, va = sbase + kOffV + st * kPfTile;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16(t_o, smem_desc(pa + (kk >> 2) * kPfTile + (kk & 3) * 32, 16, 1024),
                     smem_desc(va + kk * 2048, 16, 1024), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&o_done[pb]);
        tc_commit(&kv_empty[st]);
      }
      if (dead) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
    }
  } else {
    // ======================= softmax / epilogue (thread = query row) =======================
    const int r = tid;
    const bool row_valid = r < rows;
    const int lim = row_valid ? min(prior + q0 + r + 1, kv_len) : 0;  // keys [0, lim) visible
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool dead = false;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      if (!dead && !mbar_wait(&s_full[sb], (j >> 1) & 1)) dead = true;
      __syncwarp();  // tcgen05.ld is warp-collective
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(tbase + sb * 128 + lane_off + c4 * 32, sr[c4]);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);

      // scale > 0 (checked on the host), so the row max is taken on raw
      // scores and scaled once; only tiles crossing the causal limit mask
      const int kbase = j * kPfN;
      const bool full_tile = kbase + kPfN <= lim;
      float mt = -INFINITY;
      if (full_tile) {
#pragma unroll
        for (int c = 0; c < 128; ++c) mt = fmaxf(mt, __uint_as_float(sr[c >> 5][c & 31]));
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (kbase + c < lim) mt = fmaxf(mt, __uint_as_float(sr[c >> 5][c & 31]));
      }
      mt *= p.scale_log2;
      float factor = 1.f;
      if (mt > m_used + 8.f) {
        factor = exp2f(m_used - mt);  // 0 while nothing was visible yet
        m_used = mt;
        l *= factor;
      }
      // O (in TMEM, warp-collective access) is rescaled for the whole warp if
      // any of its rows needs it; rows that do not use factor 1
      const bool rescale = __any_sync(0xffffffffu, factor != 1.f) && j > 0;
      const float nm = (m_used == -INFINITY) ? 0.f : -m_used;
      const float sl2 = p.scale_log2;
      uint32_t pk[64];
      float lsum = 0.f;
      if (full_tile) {
#pragma unroll
        for (int c2 = 0; c2 < 64; ++c2) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(sr[(2 * c2) >> 5][(2 * c2) & 31]), sl2, nm));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sr[(2 * c2 + 1) >> 5][(2 * c2 + 1) & 31]), sl2, nm));
          lsum += p0 + p1;
          pk[c2] = pack2<T>(p0, p1);
        }
      } else {
#pragma unroll
        for (int c2 = 0; c2 < 64; ++c2) {
          const int c = 2 * c2;
          const float p0 = kbase + c < lim ? ex2_approx(fmaf(__uint_as_float(sr[c >> 5][c & 31]), sl2, nm)) : 0.f;
          const float p1 = kbase + c + 1 < lim ? ex2_approx(fmaf(__uint_as_float(sr[(c + 1) >> 5][(c + 1) & 31]), sl2, nm)) : 0.f;
          lsum += p0 + p1;
          pk[c2] = pack2<T>(p0, p1);
        }
      }
      l += lsum;
      // P buffer sb was last read by PV_{j-2}; O must be current before a rescale
      if (j >= 2 && !dead && !mbar_wait(&o_done[sb], ((j >> 1) - 1) & 1)) dead = true;
      if (rescale) {
        if (!dead && !mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1)) dead = true;
        __syncwarp();
        tc_fence_after();
#pragma unroll
        for (int c2 = 0; c2 < 2; ++c2) {
          uint32_t orr[32];
          tmem_ld32(t_o + lane_off + c2 * 32, orr);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * factor);
          tmem_st32(t_o + lane_off + c2 * 32, orr);
        }
        tmem_wait_st();
      }
      // row r of P: two 64-key sub-tiles of 128-byte swizzled rows
      uint8_t* prow = base + kOffP + sb * 2 * kPfTile + r * 128;
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          const int w = sub * 32 + c16 * 4;
          *reinterpret_cast<uint4*>(prow + sub * kPfTile + ((c16 ^ (r & 7)) << 4)) =
              make_uint4(pk[w], pk[w + 1], pk[w + 2], pk[w + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
    }
    // ---- epilogue: O / l -> out
    const int lastb = (n_tiles - 1) & 1;
    if (!dead && !mbar_wait(&o_done[lastb], ((n_tiles - 1) >> 1) & 1)) dead = true;
    __syncwarp();
    tc_fence_after();
    uint32_t o0[32], o1[32];
    tmem_ld32(t_o + lane_off, o0);
    tmem_ld32(t_o + lane_off + 32, o1);
    tmem_wait_ld();
    if (dead && r == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
    if (row_valid) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(q_begin + q0 + r) * p.out_stride +
                static_cast<int64_t>(h) * 64;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const uint32_t* src = c8 < 4 ? o0 + c8 * 8 : o1 + (c8 - 4) * 8;
        uint4 v;
        v.x = pack2<T>(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
        v.y = pack2<T>(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
        v.z = pack2<T>(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
        v.w = pack2<T>(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
        *reinterpret_cast<uint4*>(orow + c8 * 8) = v;
      }
    }
  }
  // ---- teardown: every tcgen05 access of this CTA is done before the dealloc
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, kPfTmemCols);
  }
}

bool prefill_fast_supported(const AttnArgs& a) {
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0; };
  return (a.dtype == PKV_DTYPE_F16 || a.dtype == PKV_DTYPE_BF16) && a.head_dim == 64 &&
         a.block_size == 16 && a.n_seqs <= 65535 && a.n_q_heads <= 65535 && a.max_query_len > 0 &&
         (a.q_stride * 2) % 16 == 0 && (a.out_stride * 2) % 16 == 0 && al(a.q, 16) &&
         al(a.out, 16) && al(a.k_pool, 16) && al(a.v_pool, 16) &&
         a.scale > 0.f && static_cast<int64_t>(a.n_tokens) + kPfM < (int64_t{1} << 31);
}

namespace {
std::mutex g_pf_mu;
bool g_pf_attr[64][2] = {};
}  // namespace

cudaError_t launch_prefill_fast(const AttnArgs& a, const CUtensorMap* qmap, const CUtensorMap* kmap,
                                const CUtensorMap* vmap, cudaStream_t stream) {
  if (a.n_seqs == 0 || a.n_tokens == 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  auto kern = a.dtype == PKV_DTYPE_F16 ? paged_prefill_tc_kernel<__half>
                                       : paged_prefill_tc_kernel<__nv_bfloat16>;
  {
    std::lock_guard<std::mutex> lk(g_pf_mu);
    const int k = a.dtype == PKV_DTYPE_F16 ? 0 : 1;
    if (dev < 64 && !g_pf_attr[dev][k]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmemBytes);
      if (e != cudaSuccess) return e;
      g_pf_attr[dev][k] = true;
    }
  }
  PrefillParams p;
  p.out = a.out;
  p.out_stride = a.out_stride;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.max_blocks = a.max_blocks;
  p.qsl = a.query_start_loc;
  p.num_prior = a.num_prior;
  p.num_blocks = a.num_blocks;
  p.n_tokens = a.n_tokens;
  p.group = a.n_q_heads / a.n_kv_heads;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.err = a.err;
  const dim3 grid((a.max_query_len + kPfM - 1) / kPfM, a.n_q_heads, a.n_seqs);
  kern<<<grid, kPfThreads, kPfSmemBytes, stream>>>(*qmap, *kmap, *vmap, p);
  return cudaGetLastError();
}

}  // namespace pkv
