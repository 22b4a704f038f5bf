// pkv_decode.cu -- paged decode attention for B200 (sm_100a), fp16 / bf16 KV.
//
// Replaces the reference's per-sequence gather + GQA attention for one new
// token (mini_engine/paged/block_manager.py:136-141 and
// mini_engine/model/qwen2.py:98-128 with num_new == 1).
//
// Design (HBM-bound: every KV byte is read exactly once):
//  * Stream-K split.  The flattened list of all sequences' KV blocks is cut
//    into equal ranges, one per pipeline (a "virtual CTA": a producer warp,
//    one consumer warp per KV head and their own ring), so lognormal context
//    lengths cannot unbalance the GPU.  A pipeline walks its range as
//    segments (one per sequence it touches).  For two KV heads one CTA per
//    SM holds 5 pipelines (the register limit of 5 one-pipeline CTAs), so a
//    launch starts 148 CTAs instead of 740 and reads the step's metadata
//    once per SM; other head counts run one pipeline per CTA.
//  * Producer warp: TMA tensor loads (cp.async.bulk.tensor, 128-byte swizzle)
//    of each 16-token block, one 16x64 tile per KV head for K and for V,
//    into a kStages-deep shared-memory ring guarded by mbarriers
//    (full: transaction bytes; empty: one arrival per consumer warp).
//  * Consumer warp h (one per KV head) runs m16n8k16 tensor-core MMAs with
//    the 16 tokens of a block as M and the G <= 8 query heads of the GQA
//    group as N: S^T = K Q^T, then O^T += V^T P^T with P^T transposed in
//    registers (movmatrix).  All 7 Qwen2 query heads of a group consume each
//    K/V tile from one shared-memory read.  Online softmax in fp32 (exp2)
//    with a lazy rescale: the reference max of a head moves only when a
//    block's max exceeds it by more than 2^8 (a warp vote), so most blocks
//    skip the O / l rescale; masks apply only to a sequence's last block.
//  * The ring is only 3 stages deep: with 3 stages, 5 CTAs per SM stay
//    resident (the register limit), and that measured faster than deeper
//    rings with fewer CTAs.  Two stages starve.
//  * Sequences fully inside one CTA's range are normalised and stored
//    directly.  A sequence split across CTAs leaves (m, l, O) partials in the
//    workspace, merged by a second small kernel (one CTA per sequence) that
//    is launched right behind the decode kernel.
//  * fp8 e4m3 pools (FP8 instantiation): the ring stage holds each head's
//    16 x 64-byte fp8 K and V tiles (row-major, unswizzled) plus the block's
//    per-(token, KV head) fp32 scales (TMA + two bulk copies).  Each lane
//    loads the fp8 bytes of its own MMA fragments straight into registers
//    (K: 2 x 16 bytes, V: 4 x 8 bytes, bank-conflict free), releases the
//    stage, and converts them there, exactly: K by cvt e4m3x2 -> f16x2 (the
//    transcendental pipe), V (fp16 build) by moving the e4m3 fields into f16
//    position on the integer pipes, which yields 2^-8 x the value (the 2^8 is
//    applied to O at the segment end).  Splitting the work between the two
//    pipes measured fastest of the four combinations.  That works
//    because the head dimension may be permuted: S sums over it, so K and Q
//    use the order in which lane t's four k-steps read 16 contiguous bytes,
//    and O's rows use the order in which lane g owns 8 contiguous dims (the
//    epilogue writes them back in natural order).  Scales are applied
//    outside the MMAs: K's to the token's scores, V's folded into P after
//    the softmax sums.
//  * Fused append (k_new != NULL).  16-bit pools: the consumer warp of each
//    KV head writes the newest token's row of its head into the staged K and
//    V tiles of the sequence's last block (after the TMA lands, before the
//    MMAs read it) and into the pool, so the producer's ring never waits on
//    an append.  fp8 pools: before loading the block that holds a
//    sequence's newest token, the producer warp writes that token's K and V
//    rows into the pool, quantised per row with their scales exactly as the
//    separate fp8 append does, then fences the generic-proxy writes against
//    its TMA read.
//  * Programmatic dependent launch chains append -> decode -> merge: each
//    kernel's prologue (context scan, block-table reads) runs before
//    griddepcontrol.wait and overlaps its predecessor; pool, q, out and
//    workspace are touched only after the wait.
#include <float.h>

#include <algorithm>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

#ifndef PKV_DEC_STAGES
#define PKV_DEC_STAGES 3
#endif
// fp8 stages carry half the bytes: a deeper ring keeps as many bytes in
// flight per SM as the 16-bit ring
#ifndef PKV_DEC_STAGES_FP8
#define PKV_DEC_STAGES_FP8 6
#endif
#ifndef PKV_DEC_MIN_CTAS
#define PKV_DEC_MIN_CTAS 3
#endif
// K/V tiles loaded with an L2 evict-first policy (read exactly once)
#ifndef PKV_DEC_EVICT_FIRST
#define PKV_DEC_EVICT_FIRST 1
#endif
// blocks of each CTA's range prefetched into L2 before griddepcontrol.wait
#ifndef PKV_DEC_PREFETCH
#define PKV_DEC_PREFETCH 3
#endif
template <bool FP8> __host__ __device__ constexpr int dec_stages() { return FP8 ? PKV_DEC_STAGES_FP8 : PKV_DEC_STAGES; }
constexpr int kDecMaxCtas = 1024;
constexpr int kDecMaxSeqs = 2048;
constexpr int kDecMinBlocksPerCta = 4;
constexpr int kDecTile = 2048;  // 16 tokens x 64 dims x 2 bytes
constexpr int kDecTile8 = 1024;  // 16 tokens x 64 dims x 1 byte (fp8)
constexpr float kLog2e = 1.4426950408889634f;
// lazy online-softmax rescale threshold (log2 domain): P <= 2^8
constexpr float kRescaleSlack = 8.f;

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
  float* part_ml;  // [2*kDecMaxCtas][ml_stride]: (m, l) per query head
  int ml_stride;   // floats per slot: 2*n_q_heads rounded up to 4 (16 bytes)
  int* err;
  // fused append: token context_lens[s] - 1 of sequence s (NULL = none)
  const uint8_t* k_new;
  const uint8_t* v_new;
  int64_t k_new_stride_b, v_new_stride_b;  // bytes between rows
  uint8_t* k_pool;
  uint8_t* v_pool;
  // fp8 pools: fp32 scale per (slot, KV head)
  const float* k_scale;
  const float* v_scale;
  // per-step schedule (NULL: derive it here): header, block prefix, clamped
  // lengths and each CTA's block ids in rows of sched_rows
  const int32_t* sched;
  int sched_rows;
  // nonzero once q / k_new / v_new are in memory (NULL: they already are)
  const int* input_ready;
  // 1: nothing this launch reads is written by the kernels just before it
  // (a later layer of one multi-layer call, with its own workspace): skip
  // griddepcontrol.wait before the main loop and wait at the end instead, so
  // the grid starts on SMs the previous layer's tail frees and still
  // completes after it
  int defer_wait;
  // 1 (the first layer of such a call): let the next kernel launch only
  // after this one's griddepcontrol.wait, so the call's later layers start
  // after everything before the call (a previous call's merge, which reads
  // the workspace sets they write) has completed
  int late_trigger;
  // merge over layers (blockIdx.y): out advances by out_layer_stride
  // elements, the partials by ws_layer_stride bytes per layer
  int64_t out_layer_stride;
  int64_t ws_layer_stride;
};

// Decode schedule (int32): kSchedHdr header words {n_seqs, total blocks,
// blocks per CTA, grid, row length, table width}, then the block prefix [n_seqs + 1], the
// clamped context lengths [n_seqs], then (16-byte aligned) CTA c's block ids
// at [c * rows, c * rows + per).
constexpr int kSchedHdr = 8;
__host__ __device__ inline int64_t sched_ids_offset(int n_seqs) {
  return (kSchedHdr + 2 * static_cast<int64_t>(n_seqs) + 1 + 3) & ~static_cast<int64_t>(3);
}
// ids capacity: grid x rows <= n_seqs * max_blocks + grid * (1 + kDecMinBlocksPerCta)
inline int64_t sched_ids_capacity(int n_seqs, int max_blocks) {
  return static_cast<int64_t>(n_seqs) * max_blocks + static_cast<int64_t>(kDecMaxCtas) * 5;
}
size_t decode_schedule_bytes(int n_seqs, int max_blocks) {
  return static_cast<size_t>(sched_ids_offset(n_seqs) + sched_ids_capacity(n_seqs, max_blocks)) * 4;
}
inline int sched_rows_for(int n_seqs, int max_blocks, int grid) {
  const int64_t cap = static_cast<int64_t>(n_seqs) * max_blocks;
  return static_cast<int>(std::max<int64_t>((cap + grid - 1) / grid, kDecMinBlocksPerCta));
}

// 16 fp8 e4m3 values -> 16 values of T (exact), low byte first
template <typename T> __device__ __forceinline__ uint32_t fp8x2_to(uint32_t two);
template <> __device__ __forceinline__ uint32_t fp8x2_to<__half>(uint32_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  return static_cast<uint32_t>(h.x) | (static_cast<uint32_t>(h.y) << 16);
}
template <> __device__ __forceinline__ uint32_t fp8x2_to<__nv_bfloat16>(uint32_t two) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two), __NV_E4M3);
  const float2 f = __half22float2(__half2(h));
  return pack2<__nv_bfloat16>(f.x, f.y);
}
// fp8 -> f16 on the integer pipes (the fp16 instantiation): the e4m3 fields
// moved into f16 position, which is the value times 2^-8 (exact, e4m3
// subnormals included: they land on f16 subnormals).  The 2^8 goes into the
// score scale (K) or into O at the segment end (V).  The NaN encodings
// 0x7f / 0xff map to +-480; the quantising append never stores them.  Takes
// conversions off the transcendental pipe, which cvt and the softmax's exp2
// share.
#ifndef PKV_FP8_ALU_CVT
#define PKV_FP8_ALU_CVT 2  // bit 0: K tiles, bit 1: V tiles (K by cvt measured faster)
#endif

template <typename T>
__device__ __forceinline__ void fp8x16_to(const uint4& in, uint4& lo, uint4& hi) {
  lo = make_uint4(fp8x2_to<T>(in.x & 0xffffu), fp8x2_to<T>(in.x >> 16), fp8x2_to<T>(in.y & 0xffffu),
                  fp8x2_to<T>(in.y >> 16));
  hi = make_uint4(fp8x2_to<T>(in.z & 0xffffu), fp8x2_to<T>(in.z >> 16), fp8x2_to<T>(in.w & 0xffffu),
                  fp8x2_to<T>(in.w >> 16));
}

size_t decode_workspace_bytes(int n_seqs, int n_q_heads, int head_dim) {
  (void)n_seqs;
  const size_t parts = static_cast<size_t>(2) * kDecMaxCtas *
                       (n_q_heads * head_dim + ((2 * n_q_heads + 3) & ~3)) * 4;
  return (parts + 255) & ~static_cast<size_t>(255);
}

// the shapes the tensor-core kernel serves (pointer alignment aside)
bool decode_fast_supported_shape(const AttnArgs& a) {
  const int G = a.n_q_heads / a.n_kv_heads;
  return (a.dtype == PKV_DTYPE_F16 || a.dtype == PKV_DTYPE_BF16) && a.head_dim == 64 &&
         a.block_size == 16 && (a.n_kv_heads == 1 || a.n_kv_heads == 2 || a.n_kv_heads == 4) &&
         G <= 8 && a.n_q_heads <= 32 && a.n_seqs <= kDecMaxSeqs;
}

bool decode_fast_supported(const AttnArgs& a) {
  const int G = a.n_q_heads / a.n_kv_heads;
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0; };
  if (a.k_new != nullptr &&
      (!al(a.k_new, 16) || !al(a.v_new, 16) || (a.k_new_stride * 2) % 16 || (a.v_new_stride * 2) % 16))
    return false;
  // fp8 pools: the scale rows are bulk-copied (16-byte aligned)
  if (a.k_scale != nullptr && (!al(a.k_scale, 16) || !al(a.v_scale, 16))) return false;
  return (a.dtype == PKV_DTYPE_F16 || a.dtype == PKV_DTYPE_BF16) && a.head_dim == 64 &&
         a.block_size == 16 && (a.n_kv_heads == 1 || a.n_kv_heads == 2 || a.n_kv_heads == 4) &&
         G <= 8 && a.n_q_heads <= 32 && a.n_seqs <= kDecMaxSeqs && (a.q_stride % 2) == 0 &&
         (a.out_stride % 4) == 0 && al(a.q, 4) && al(a.out, 8) && al(a.k_pool, 16) &&
         al(a.v_pool, 16);
}

// exclusive scan of n values in smem (in place); returns the total to all threads
__device__ __forceinline__ int block_exclusive_scan(int* vals, int n, int* scratch) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int per = (n + nt - 1) / nt;
  const int lo = min(n, tid * per), hi = min(n, lo + per);
  int sum = 0;
  for (int i = lo; i < hi; ++i) sum += vals[i];
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

// Q^T fragments of this warp's GQA group, in the dim order of the K
// fragments (QL): 0 natural, qa[kk] = Q[head g][16kk + 2t (+8)]; 1 (fp8,
// cvt) k-step kk's k indices 2t, 2t + 1, 2t + 8, 2t + 9 are dims
// 16t + 4kk + {0, 1, 2, 3}; 2 (fp8, integer-pipe conversion) they are dims
// 16t + 4kk + {0, 2, 1, 3}
template <typename T, int QL>
__device__ __forceinline__ void load_q_frag(uint32_t (&qa)[4][2], const DecodeParams& p, int s,
                                            int h, int lane) {
  const int g = lane >> 2, t = lane & 3;
  if (g < p.group) {
    const T* row = static_cast<const T*>(p.q) + static_cast<int64_t>(s) * p.q_stride +
                   static_cast<int64_t>(h * p.group + g) * 64;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int d0 = QL ? 16 * t + 4 * kk : 16 * kk + 2 * t;
      const int d1 = QL ? d0 + 2 : d0 + 8;
      const uint32_t u0 = __ldg(reinterpret_cast<const uint32_t*>(row + d0));
      const uint32_t u1 = __ldg(reinterpret_cast<const uint32_t*>(row + d1));
      qa[kk][0] = QL == 2 ? __byte_perm(u0, u1, 0x5410) : u0;
      qa[kk][1] = QL == 2 ? __byte_perm(u0, u1, 0x7632) : u1;
    }
  } else {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) qa[kk][0] = qa[kk][1] = 0u;
  }
}

// workspace slot of CTA c's partial for a sequence whose blocks start at blk_lo
__device__ __forceinline__ int partial_slot(int c, int per, int blk_lo) {
  return (blk_lo > c * per) ? 2 * c + 1 : 2 * c;
}

template <typename T, int NKV, bool FP8, int PIPES>
__global__ void __launch_bounds__(32 * (NKV + 1) * PIPES, PIPES > 1 ? 1 : PKV_DEC_MIN_CTAS)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const DecodeParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int nkv = NKV;
  const int B = p.n_seqs;
  // PIPES independent pipelines (a producer warp and nkv consumer warps each,
  // with their own ring) per CTA, each serving one stream-K range (a
  // "virtual CTA"): one CTA per SM starts all of them together and does the
  // metadata prologue once
  constexpr int kPw = NKV + 1;
  const int pipe = warp / kPw;
  const int pwarp = warp - pipe * kPw;
  const int vcta = blockIdx.x * PIPES + pipe;
  const int vgrid = gridDim.x * PIPES;

  // ---- shared memory carve-up (tiles 1024-byte aligned for the 128B swizzle)
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  // stage: K tiles, V tiles (fp8: then the K and V scale rows of the block)
  constexpr int kDecStages = dec_stages<FP8>();
  constexpr int tile_bytes = FP8 ? kDecTile8 : kDecTile;
  constexpr int scale_bytes = FP8 ? 16 * nkv * 4 : 0;
  constexpr int stage_bytes = 2 * nkv * tile_bytes + 2 * scale_bytes;
  uint8_t* tiles = base + pipe * (kDecStages * stage_bytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + PIPES * (kDecStages * stage_bytes));
  uint64_t* full_bar = bars + pipe * (2 * kDecStages);
  uint64_t* empty_bar = full_bar + kDecStages;
  int* misc = reinterpret_cast<int*>(bars + PIPES * (2 * kDecStages));  // [1..33]: scan scratch
  int* prefix = misc + 40;                           // [B+1]
  int* ctxs = prefix + (B + 1);                      // [B]

  // ---- prologue (reads only metadata)
  int total, per;
  int sched_id0 = 0;  // producer lanes: this CTA's first 32 block ids (schedule)
  if (p.sched != nullptr) {
    // the step's schedule: one round trip, no scan; the producer's first
    // block ids are loaded in the same round trip
    const int32_t* sp = p.sched + kSchedHdr;
    for (int s = tid; s <= B; s += blockDim.x) prefix[s] = __ldg(sp + s);
    for (int s = tid; s < B; s += blockDim.x) ctxs[s] = __ldg(sp + B + 1 + s);
    if (pwarp == nkv && lane < p.sched_rows)
      sched_id0 = __ldg(p.sched + sched_ids_offset(B) + static_cast<int64_t>(vcta) * p.sched_rows + lane);
    total = __ldg(p.sched + 1);
    per = __ldg(p.sched + 2);
    // a schedule built for another batch, grid or table width (its row
    // length and size follow from the width) is not read
    if (__ldg(p.sched) != B || __ldg(p.sched + 3) != vgrid || __ldg(p.sched + 4) != p.sched_rows ||
        __ldg(p.sched + 5) != p.max_blocks) {
      // a schedule built for another batch or grid: do nothing
      if (tid == 0 && vcta == 0) raise_flag(p.err, PKV_FLAG_BAD_SCHEDULE);
      if (p.defer_wait || p.late_trigger) pdl_wait();
      if (tid == 0) pdl_trigger();
      return;
    }
    __syncthreads();
  } else {
    // clamp contexts, prefix-sum block counts
    const int cap_tokens = p.max_blocks * 16;
    for (int s = tid; s < B; s += blockDim.x) {
      int c = p.context_lens[s];
      if (c < 0) c = 0;
      if (c > cap_tokens) {
        if (vcta == 0) raise_flag(p.err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
        c = cap_tokens;
      }
      ctxs[s] = c;
      prefix[s] = (c + 15) >> 4;
    }
    __syncthreads();
    total = block_exclusive_scan(prefix, B, misc + 1);
    if (tid == 0) prefix[B] = total;
    __syncthreads();
    per = max((total + vgrid - 1) / vgrid, kDecMinBlocksPerCta);
  }
  const int n_active = (total + per - 1) / per;
  const bool active = vcta < n_active;

  // the merge kernel behind this one may be scheduled now: it waits for this
  // grid's completion before it reads anything this grid writes
  if (tid == 0 && !p.late_trigger) pdl_trigger();

  if (tid == 0) {
    for (int i = 0; i < PIPES * 2 * kDecStages; ++i)
      mbar_init(&bars[i], (i % (2 * kDecStages)) < kDecStages ? 1 : nkv);
    fence_barrier_init();
  }
  __syncthreads();
  if (!active) {
    if (p.defer_wait || p.late_trigger) pdl_wait();
    if (p.late_trigger && tid == 0) pdl_trigger();
    return;
  }

  const int r0 = vcta * per;
  const int r1 = min(r0 + per, total);

  if (pwarp == nkv) {
    // ======================= producer warp =======================
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    bool dead = false, waited = false;
#if PKV_DEC_EVICT_FIRST
    const uint64_t kv_policy = l2_evict_first_policy();
#endif
    int i = 0;
    for (int b0 = r0; b0 < r1; b0 += 32) {
      const int gb = b0 + lane;
      int id = 0;
      int app_seq = -1, app_row = 0;  // fused append: this block holds seq's newest token
      if (gb < r1) {
        const int s = find_seq(prefix, B, gb);
        const int jb = gb - prefix[s];
        if (p.sched != nullptr) {
          // validated by the schedule builder (a bad id is stored as -1)
          id = b0 == r0 ? sched_id0
                        : __ldg(p.sched + sched_ids_offset(B) +
                                static_cast<int64_t>(vcta) * p.sched_rows + (gb - r0));
        } else {
          id = __ldg(p.block_tables + static_cast<int64_t>(s) * p.bt_stride + jb);
          if (id < 0 || id >= p.num_blocks) {
            raise_flag(p.err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
            id = -1;
          }
        }
        if (id < 0) {
          id = 0;  // read a valid block; never write through a bad id
        } else if (FP8 && p.k_new != nullptr && gb == prefix[s + 1] - 1) {
          app_seq = s;  // 16-bit pools: the consumers append (see below)
          app_row = id * 16 + ((ctxs[s] - 1) & 15);
        }
      }
      if (!waited) {
        // warm L2 with the first blocks' K/V while the preceding kernel ends
        if (gb < r1 && lane < PKV_DEC_PREFETCH) {
          prefetch_l2(p.k_pool + static_cast<int64_t>(id) * (nkv * tile_bytes), nkv * tile_bytes);
          prefetch_l2(p.v_pool + static_cast<int64_t>(id) * (nkv * tile_bytes), nkv * tile_bytes);
        }
        if (!p.defer_wait) pdl_wait();  // the pool may still be written by the preceding kernel
        waited = true;
      }
      const int n = min(32, r1 - b0);
      // fused append, fp8 pools: the warp writes the quantised K and V rows
      // (with their scales) of the sequence whose newest token lies in batch
      // block kk; fence_appends() then orders those generic-proxy writes
      // before lane 0's TMA reads
      auto append_rows = [&](int kk) {
        const int a_seq = __shfl_sync(0xffffffffu, app_seq, kk);
        const int row = __shfl_sync(0xffffffffu, app_row, kk);
        fp8_store_token<T>(reinterpret_cast<const T*>(p.k_new + a_seq * p.k_new_stride_b),
                           p.k_pool + static_cast<int64_t>(row) * (nkv * 64),
                           const_cast<float*>(p.k_scale) + static_cast<int64_t>(row) * nkv, nkv, 64,
                           lane);
        fp8_store_token<T>(reinterpret_cast<const T*>(p.v_new + a_seq * p.v_new_stride_b),
                           p.v_pool + static_cast<int64_t>(row) * (nkv * 64),
                           const_cast<float*>(p.v_scale) + static_cast<int64_t>(row) * nkv, nkv, 64,
                           lane);
      };
      auto fence_appends = [&]() {
        fence_proxy_async_global();
        __syncwarp();
        if (lane == 0) fence_proxy_async_global();
      };
      // batch blocks that hold a sequence's newest token and are not yet written
      uint32_t pending = FP8 ? __ballot_sync(0xffffffffu, app_seq >= 0) : 0u;
      for (int k = 0; k < n; ++k, ++i) {
        const int blk = __shfl_sync(0xffffffffu, id, k);
        if ((pending >> k) & 1u) {  // append before the block is loaded
          append_rows(k);
          fence_appends();
          pending &= ~(1u << k);
        }
        if (lane == 0 && !dead) {
          const int st = i % kDecStages;
          if (!mbar_wait(&empty_bar[st], ((i / kDecStages) & 1) ^ 1)) {
            raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
            dead = true;
          } else {
            uint8_t* stg = tiles + st * stage_bytes;
            mbar_arrive_expect_tx(&full_bar[st], stage_bytes);
#pragma unroll
            for (int hk = 0; hk < nkv; ++hk) {
#if PKV_DEC_EVICT_FIRST
              tma_load_3d_hint(stg + hk * tile_bytes, &kmap, &full_bar[st], 0, hk, blk * 16, kv_policy);
              tma_load_3d_hint(stg + (nkv + hk) * tile_bytes, &vmap, &full_bar[st], 0, hk, blk * 16,
                               kv_policy);
#else
              tma_load_3d(stg + hk * tile_bytes, &kmap, &full_bar[st], 0, hk, blk * 16);
              tma_load_3d(stg + (nkv + hk) * tile_bytes, &vmap, &full_bar[st], 0, hk, blk * 16);
#endif
            }
            if constexpr (FP8) {
              bulk_load(stg + 2 * nkv * tile_bytes, p.k_scale + static_cast<int64_t>(blk) * 16 * nkv,
                        scale_bytes, &full_bar[st]);
              bulk_load(stg + 2 * nkv * tile_bytes + scale_bytes,
                        p.v_scale + static_cast<int64_t>(blk) * 16 * nkv, scale_bytes, &full_bar[st]);
            }
          }
        }
      }
    }
    if (p.defer_wait) pdl_wait();  // complete only after the kernel before this one
    return;
  }

  // ======================= consumer warps (warp = kv head) =======================
  // Fragment layout (m16n8k16): g = lane / 4, t = lane % 4.
  //   S^T = K Q^T   : A = K tile (16 tokens x 16 dims per k-step, ldmatrix),
  //                   B = Q^T (16 dims x 8 heads; heads >= G are zero),
  //                   C holds tokens {g, g+8} x heads {2t, 2t+1}.
  //   O^T += V^T P^T: A = V^T (16 dims x 16 tokens, ldmatrix.trans) per
  //                   16-dim tile, B = P^T from C via movmatrix.trans,
  //                   C holds dims {16mt+g, 16mt+g+8} x heads {2t, 2t+1}.
  if (!p.defer_wait) pdl_wait();
  if (p.late_trigger && tid == 0) pdl_trigger();  // thread 0 is a consumer lane of pipeline 0
  if (p.input_ready != nullptr) {
    // inputs that a copy on another stream brings in: one lane waits for the
    // word the copy engine sets after them, then the warp reads them
    int ok = 1;
    if (lane == 0) ok = wait_word_nonzero(p.input_ready);
    if (!__shfl_sync(0xffffffffu, ok, 0) && lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
    __syncwarp();
  }
  const int h = pwarp;
  const int g = lane >> 2, t = lane & 3;
  // fp8 conversion on the integer pipes (fp16) or by cvt (bf16)
  constexpr bool kF16 = std::is_same<T, __half>::value;
  constexpr bool kAluK = FP8 && kF16 && (PKV_FP8_ALU_CVT & 1);
  constexpr bool kAluV = FP8 && kF16 && (PKV_FP8_ALU_CVT & 2);
  constexpr int QL = !FP8 ? 0 : kAluK ? 2 : 1;
  // the integer conversion yields 2^-8 x the e4m3 values: K's 2^8 goes into
  // the score scale, V's into O at the segment epilogue
  constexpr float kCvt = kAluV ? 256.f : 1.f;
  const float sl2 = p.scale_log2 * (kAluK ? 256.f : 1.f);
  // fp8 V byte interleave (tokens 2t / 2t + 1 of dims 8g + 2mt, + 1); lanes
  // with sw = 1 loaded the token pair swapped, so their operands swap back
  const int sw = t & 1;
  const uint32_t sel_flip = sw ? 0x4444u : 0u;
  const uint32_t sel_lo = (kAluV ? 0x5410u : 0x5140u) ^ sel_flip;  // even mt
  const uint32_t sel_hi = (kAluV ? 0x7632u : 0x7362u) ^ sel_flip;  // odd mt
  const int G = p.group;
  const bool ok0 = 2 * t < G, ok1 = 2 * t + 1 < G;  // this lane's two heads exist
  const int qh0 = h * G + 2 * t;                    // its first query head
  bool dead = false;

  int s = find_seq(prefix, B, r0);
  uint32_t qa[4][2];
  load_q_frag<T, QL>(qa, p, s, h, lane);
  int pos = r0;
  int i = 0;
  while (pos < r1) {
    const int seg_end = min(prefix[s + 1], r1);
    const int jb0 = pos - prefix[s];
    const bool complete = prefix[s] >= r0 && prefix[s + 1] <= r1;
    int s_next = s + 1;
    while (s_next < B && prefix[s_next + 1] == prefix[s_next]) ++s_next;
    uint32_t qn[4][2];
    if (seg_end < r1) load_q_frag<T, QL>(qn, p, s_next, h, lane);

    const int ctx = ctxs[s];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

    const int jb_end = jb0 + (seg_end - pos);
    if constexpr (FP8) {
      // Two ring blocks per iteration (32 tokens): two independent QK^T
      // chains, one max reduction / vote / rescale for both, and the PV
      // products of both interleaved.  An odd last block is paired with a
      // phantom block (no wait, zero fragments, every token masked: P = 0).
      struct Frag {
        uint4 kr0, kr1;  // K rows g and g + 8, bytes 16t .. 16t + 15
        uint2 vr[4];     // V rows 2t + sw, 2t + 1 - sw, 2t + 8 + sw, 2t + 9 - sw
        float ks0, ks1, vs0, vs1;  // scales of tokens g, g + 8
        int valid;       // tokens of the block inside the context
      };
      auto load = [&](int ii, int jbb, Frag& f) {
        const int st = ii % kDecStages;
        if (!dead && !mbar_wait(&full_bar[st], (ii / kDecStages) & 1)) {
          if (lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
          dead = true;
        }
        // only a sequence's last block has fewer than 16 tokens (warp-uniform)
        f.valid = min(16, ctx - jbb * 16);
        const uint8_t* stg = tiles + st * stage_bytes;
        const uint8_t* k8 = stg + h * kDecTile8;
        const uint8_t* v8 = stg + (nkv + h) * kDecTile8;
        const float* ksc = reinterpret_cast<const float*>(stg + 2 * nkv * kDecTile8);
        const float* vsc = ksc + 16 * nkv;
        f.kr0 = *reinterpret_cast<const uint4*>(k8 + g * 64 + t * 16);
        f.kr1 = *reinterpret_cast<const uint4*>(k8 + (g + 8) * 64 + t * 16);
        // lanes with odd t (sw = 1) take their row pair in the other order, so
        // that each 8-byte load's 32 lanes fill all 32 banks (two wavefronts);
        // the byte permutes below swap their operands back (sel ^ 0x4444)
        f.vr[0] = *reinterpret_cast<const uint2*>(v8 + (2 * t + sw) * 64 + 8 * g);
        f.vr[1] = *reinterpret_cast<const uint2*>(v8 + (2 * t + 1 - sw) * 64 + 8 * g);
        f.vr[2] = *reinterpret_cast<const uint2*>(v8 + (2 * t + 8 + sw) * 64 + 8 * g);
        f.vr[3] = *reinterpret_cast<const uint2*>(v8 + (2 * t + 9 - sw) * 64 + 8 * g);
        f.ks0 = ksc[g * nkv + h];
        f.ks1 = ksc[(g + 8) * nkv + h];
        f.vs0 = vsc[g * nkv + h];
        f.vs1 = vsc[(g + 8) * nkv + h];
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[st]);  // the stage is free once in registers
        if (f.valid < 16) {
          // rows past the context: scales 0, V bytes 0 (an unused slot may hold
          // any bytes, and 0 x NaN would reach O); their scores are masked below
          if (g >= f.valid) f.ks0 = f.vs0 = 0.f;
          if (g + 8 >= f.valid) f.ks1 = f.vs1 = 0.f;
          const uint2 z = make_uint2(0u, 0u);
          if (2 * t + sw >= f.valid) f.vr[0] = z;
          if (2 * t + 1 - sw >= f.valid) f.vr[1] = z;
          if (2 * t + 8 + sw >= f.valid) f.vr[2] = z;
          if (2 * t + 9 - sw >= f.valid) f.vr[3] = z;
        }
      };
      // S^T = K Q^T (16 tokens x 8 heads), 4 k-steps of 16 dims
      auto qk = [&](const Frag& f, float (&sc)[4]) {
        sc[0] = sc[1] = sc[2] = sc[3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          // k-step kk: bytes 4kk .. 4kk + 3 of rows g and g + 8
          const uint32_t w0 = kk == 0 ? f.kr0.x : kk == 1 ? f.kr0.y : kk == 2 ? f.kr0.z : f.kr0.w;
          const uint32_t w1 = kk == 0 ? f.kr1.x : kk == 1 ? f.kr1.y : kk == 2 ? f.kr1.z : f.kr1.w;
          uint32_t a[4];
          if constexpr (kAluK) {
            a[0] = e4m3_even_h2(w0);
            a[1] = e4m3_even_h2(w1);
            a[2] = e4m3_odd_h2(w0);
            a[3] = e4m3_odd_h2(w1);
          } else {
            a[0] = fp8x2_to<T>(w0 & 0xffffu);
            a[1] = fp8x2_to<T>(w1 & 0xffffu);
            a[2] = fp8x2_to<T>(w0 >> 16);
            a[3] = fp8x2_to<T>(w1 >> 16);
          }
          mma16816<T>(sc, a, qa[kk][0], qa[kk][1]);
        }
      };
      // O^T += V^T P^T, 4 tiles of 16 dims (O rows g, g + 8 of tile mt are
      // dims 8g + 2mt and 8g + 2mt + 1)
      auto pv_a = [&](const Frag& f, int mt, uint32_t (&a)[4]) {
        // interleave tokens (2t, 2t + 1) and (2t + 8, 2t + 9) byte by byte
        const uint32_t sel = (mt & 1) ? sel_hi : sel_lo;
        const uint32_t x01 = __byte_perm(mt < 2 ? f.vr[0].x : f.vr[0].y, mt < 2 ? f.vr[1].x : f.vr[1].y, sel);
        const uint32_t x23 = __byte_perm(mt < 2 ? f.vr[2].x : f.vr[2].y, mt < 2 ? f.vr[3].x : f.vr[3].y, sel);
        if constexpr (kAluV) {
          a[0] = e4m3_even_h2(x01);
          a[1] = e4m3_odd_h2(x01);
          a[2] = e4m3_even_h2(x23);
          a[3] = e4m3_odd_h2(x23);
        } else {
          a[0] = fp8x2_to<T>(x01 & 0xffffu);
          a[1] = fp8x2_to<T>(x01 >> 16);
          a[2] = fp8x2_to<T>(x23 & 0xffffu);
          a[3] = fp8x2_to<T>(x23 >> 16);
        }
      };
      for (int jb = jb0; jb < jb_end; jb += 2) {
        const bool two = jb + 1 < jb_end;
        Frag fa, fb;
        load(i, jb, fa);
        if (two) {
          load(i + 1, jb + 1, fb);
        } else {
          fb.kr0 = fb.kr1 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int r = 0; r < 4; ++r) fb.vr[r] = make_uint2(0u, 0u);
          fb.ks0 = fb.ks1 = fb.vs0 = fb.vs1 = 0.f;
          fb.valid = 0;
        }
        i += two ? 2 : 1;
        float sa_[4], sb_[4];
        qk(fa, sa_);
        qk(fb, sb_);
        // ---- online softmax per head over the 32 tokens (exp2 domain).  A
        // lane's two heads (2t, 2t + 1) of one token are a pair for the
        // paired fp32 instructions of sm_100 (each lane rounded as the scalar
        // instruction rounds it)
        const float ka0 = sl2 * fa.ks0, ka1 = sl2 * fa.ks1, kb0 = sl2 * fb.ks0, kb1 = sl2 * fb.ks1;
        float2 xa01 = __fmul2_rn(make_float2(sa_[0], sa_[1]), make_float2(ka0, ka0));  // block a, token g
        float2 xa23 = __fmul2_rn(make_float2(sa_[2], sa_[3]), make_float2(ka1, ka1));  // block a, token g + 8
        float2 xb01 = __fmul2_rn(make_float2(sb_[0], sb_[1]), make_float2(kb0, kb0));
        float2 xb23 = __fmul2_rn(make_float2(sb_[2], sb_[3]), make_float2(kb1, kb1));
        const float2 ninf = make_float2(-INFINITY, -INFINITY);
        if (fa.valid < 16) {
          if (g >= fa.valid) xa01 = ninf;
          if (g + 8 >= fa.valid) xa23 = ninf;
        }
        if (fb.valid < 16) {
          if (g >= fb.valid) xb01 = ninf;
          if (g + 8 >= fb.valid) xb23 = ninf;
        }
        float ma = fmaxf(fmaxf(xa01.x, xa23.x), fmaxf(xb01.x, xb23.x));
        float mb = fmaxf(fmaxf(xa01.y, xa23.y), fmaxf(xb01.y, xb23.y));
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, off));
          mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
        }
        // lazy rescale: the reference max moves only when some head's max
        // exceeds it by more than kRescaleSlack, so P stays <= 2^kRescaleSlack
        // and the (m, l, O) triple stays exact relative to its own m
        if (__any_sync(0xffffffffu, ma > m0 + kRescaleSlack || mb > m1 + kRescaleSlack)) {
          const float mna = fmaxf(m0, ma), mnb = fmaxf(m1, mb);
          const float ca = ex2_approx(m0 - mna), cb = ex2_approx(m1 - mnb);
          l0 *= ca;
          l1 *= cb;
#pragma unroll
          for (int j = 0; j < 4; ++j) { o[j][0] *= ca; o[j][1] *= cb; o[j][2] *= ca; o[j][3] *= cb; }
          m0 = mna;
          m1 = mnb;
        }
        const float2 nm = make_float2(-m0, -m1);
        const float2 da01 = __fadd2_rn(xa01, nm), da23 = __fadd2_rn(xa23, nm);
        const float2 db01 = __fadd2_rn(xb01, nm), db23 = __fadd2_rn(xb23, nm);
        const float2 pa01 = make_float2(ex2_approx(da01.x), ex2_approx(da01.y));
        const float2 pa23 = make_float2(ex2_approx(da23.x), ex2_approx(da23.y));
        const float2 pb01 = make_float2(ex2_approx(db01.x), ex2_approx(db01.y));
        const float2 pb23 = make_float2(ex2_approx(db23.x), ex2_approx(db23.y));
        // l += (pa(g) + pa(g + 8)) + (pb(g) + pb(g + 8)), per head
        const float2 ls = __fadd2_rn(__fadd2_rn(pa01, pa23), __fadd2_rn(pb01, pb23));
        l0 += ls.x;
        l1 += ls.y;
        // P^T fragments with V's per-token scale folded in (l sums the unscaled P)
        const float2 qa01 = __fmul2_rn(pa01, make_float2(fa.vs0, fa.vs0));
        const float2 qa23 = __fmul2_rn(pa23, make_float2(fa.vs1, fa.vs1));
        const float2 qb01 = __fmul2_rn(pb01, make_float2(fb.vs0, fb.vs0));
        const float2 qb23 = __fmul2_rn(pb23, make_float2(fb.vs1, fb.vs1));
        const uint32_t ba0 = movmatrix_t(pack2<T>(qa01.x, qa01.y));  // tokens 0-7
        const uint32_t ba1 = movmatrix_t(pack2<T>(qa23.x, qa23.y));  // tokens 8-15
        const uint32_t bb0 = movmatrix_t(pack2<T>(qb01.x, qb01.y));
        const uint32_t bb1 = movmatrix_t(pack2<T>(qb23.x, qb23.y));
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          uint32_t aa[4], ab[4];
          pv_a(fa, mt, aa);
          pv_a(fb, mt, ab);
          mma16816<T>(o[mt], aa, ba0, ba1);
          mma16816<T>(o[mt], ab, bb0, bb1);
        }
      }
    } else {
    // Fused append, 16-bit pools: the segment that ends a sequence holds its
    // newest token (row ctx - 1).  This warp, the only reader of its KV
    // head's tiles, loads the head's new K and V values now (4 bytes a
    // lane), writes them into the staged tiles of the last block once its
    // TMA has landed (the slot's old bytes are overwritten before any
    // ldmatrix reads them) and stores them to the pool.  The producer never
    // waits on the append; whether its TMA read of the slot sees the old or
    // the new bytes, the tile the MMAs read holds the new row.
    const bool app = p.k_new != nullptr && seg_end == prefix[s + 1];
    uint32_t kn = 0u, vn = 0u;
    int app_id = -1;
    if (app) {
      kn = __ldg(reinterpret_cast<const uint32_t*>(p.k_new + s * p.k_new_stride_b + h * 128) + lane);
      vn = __ldg(reinterpret_cast<const uint32_t*>(p.v_new + s * p.v_new_stride_b + h * 128) + lane);
      const int gl = prefix[s + 1] - 1;  // the sequence's last block in the step's order
      if (p.sched != nullptr) {
        // validated by the schedule builder (a bad id is stored as -1)
        app_id = __ldg(p.sched + sched_ids_offset(B) + static_cast<int64_t>(vcta) * p.sched_rows + (gl - r0));
      } else {
        app_id = __ldg(p.block_tables + static_cast<int64_t>(s) * p.bt_stride + (gl - prefix[s]));
        if (app_id >= p.num_blocks) app_id = -1;  // flagged by the producer
      }
    }
    for (int jb = jb0; jb < jb_end; ++jb, ++i) {
      const int st = i % kDecStages;
      if (!dead && !mbar_wait(&full_bar[st], (i / kDecStages) & 1)) {
        if (lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
        dead = true;
      }
      // tokens of this block inside the context; only a sequence's last
      // block has fewer than 16 (warp-uniform)
      const int valid = min(16, ctx - jb * 16);
      const uint32_t kt = smem_u32(tiles + st * stage_bytes + h * kDecTile);
      const uint32_t vt = smem_u32(tiles + st * stage_bytes + (nkv + h) * kDecTile);
      const bool patch = app && jb == jb_end - 1;  // warp-uniform
      if (patch) {
        // row valid - 1 of the 128B-swizzled tiles: 16-byte chunk c of row r
        // sits at chunk c ^ (r & 7); lane l holds bytes 4l .. 4l + 3
        const int r = valid - 1;
        const int off = r * 128 + (((lane >> 2) ^ (r & 7)) << 4) + (lane & 3) * 4;
        *reinterpret_cast<uint32_t*>(tiles + st * stage_bytes + h * kDecTile + off) = kn;
        *reinterpret_cast<uint32_t*>(tiles + st * stage_bytes + (nkv + h) * kDecTile + off) = vn;
        __syncwarp();
      }
      // ---- S^T = K Q^T (16 tokens x 8 heads), 4 k-steps of 16 dims
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
      const int mi = lane >> 3;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        const int row = (lane & 7) + ((mi & 1) << 3);
        const int chunk = 2 * kk + (mi >> 1);
        ldsm_x4(kt + row * 128 + ((chunk ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
        mma16816<T>(sc, a, qa[kk][0], qa[kk][1]);
      }
      // ---- online softmax per head (exp2 domain)
      float x0 = sc[0] * sl2, x1 = sc[1] * sl2;  // token g
      float x2 = sc[2] * sl2, x3 = sc[3] * sl2;  // token g + 8
      if (valid < 16) {
        if (g >= valid) x0 = x1 = -INFINITY;
        if (g + 8 >= valid) x2 = x3 = -INFINITY;
      }
      float ma = fmaxf(x0, x2), mb = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        ma = fmaxf(ma, __shfl_xor_sync(0xffffffffu, ma, off));
        mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, off));
      }
      // lazy rescale: the reference max moves only when some head's block max
      // exceeds it by more than kRescaleSlack, so P stays <= 2^kRescaleSlack
      // and the (m, l, O) triple stays exact relative to its own m
      if (__any_sync(0xffffffffu, ma > m0 + kRescaleSlack || mb > m1 + kRescaleSlack)) {
        const float mna = fmaxf(m0, ma), mnb = fmaxf(m1, mb);
        const float ca = ex2_approx(m0 - mna), cb = ex2_approx(m1 - mnb);
        l0 *= ca;
        l1 *= cb;
#pragma unroll
        for (int j = 0; j < 4; ++j) { o[j][0] *= ca; o[j][1] *= cb; o[j][2] *= ca; o[j][3] *= cb; }
        m0 = mna;
        m1 = mnb;
      }
      const float p0 = ex2_approx(x0 - m0), p2 = ex2_approx(x2 - m0);
      const float p1 = ex2_approx(x1 - m1), p3 = ex2_approx(x3 - m1);
      l0 += p0 + p2;
      l1 += p1 + p3;
      // ---- P^T fragments: transpose (token x head) 8x8 tiles to (head x token)
      const uint32_t b0 = movmatrix_t(pack2<T>(p0, p1));  // tokens 0-7
      const uint32_t b1 = movmatrix_t(pack2<T>(p2, p3));  // tokens 8-15
      // ---- O^T += V^T P^T, 4 tiles of 16 dims
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        uint32_t a[4];
        const int row = (lane & 7) + ((mi >> 1) << 3);
        const int chunk = 2 * mt + (mi & 1);
        ldsm_x4_t(vt + row * 128 + ((chunk ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
        mma16816<T>(o[mt], a, b0, b1);
      }
      // the patched row's generic writes before the stage's next TMA write
      if (patch) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_bar[st]);
    }
    if (app_id >= 0) {  // the new row into the pool (its slot of the last block)
      const int64_t row = static_cast<int64_t>(app_id) * 16 + ((ctx - 1) & 15);
      reinterpret_cast<uint32_t*>(p.k_pool + (row * nkv + h) * 128)[lane] = kn;
      reinterpret_cast<uint32_t*>(p.v_pool + (row * nkv + h) * 128)[lane] = vn;
    }
    }

    // ---- segment epilogue: per-head sums over the 8 token groups
    float lt0 = l0, lt1 = l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      lt0 += __shfl_xor_sync(0xffffffffu, lt0, off);
      lt1 += __shfl_xor_sync(0xffffffffu, lt1, off);
    }
    if (complete) {
      T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(s) * p.out_stride +
                static_cast<int64_t>(qh0) * 64;
      const float i0 = kCvt / lt0, i1 = kCvt / lt1;
      if constexpr (FP8) {
        // this lane holds dims 8g .. 8g + 7 of heads 2t and 2t + 1
        if (ok0) {
          *reinterpret_cast<uint2*>(orow + 8 * g) =
              make_uint2(pack2<T>(o[0][0] * i0, o[0][2] * i0), pack2<T>(o[1][0] * i0, o[1][2] * i0));
          *reinterpret_cast<uint2*>(orow + 8 * g + 4) =
              make_uint2(pack2<T>(o[2][0] * i0, o[2][2] * i0), pack2<T>(o[3][0] * i0, o[3][2] * i0));
        }
        if (ok1) {
          *reinterpret_cast<uint2*>(orow + 64 + 8 * g) =
              make_uint2(pack2<T>(o[0][1] * i1, o[0][3] * i1), pack2<T>(o[1][1] * i1, o[1][3] * i1));
          *reinterpret_cast<uint2*>(orow + 64 + 8 * g + 4) =
              make_uint2(pack2<T>(o[2][1] * i1, o[2][3] * i1), pack2<T>(o[3][1] * i1, o[3][3] * i1));
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          if (ok0) {
            orow[16 * mt + g] = Elem<T>::from_f(o[mt][0] * i0);
            orow[16 * mt + g + 8] = Elem<T>::from_f(o[mt][2] * i0);
          }
          if (ok1) {
            orow[64 + 16 * mt + g] = Elem<T>::from_f(o[mt][1] * i1);
            orow[64 + 16 * mt + g + 8] = Elem<T>::from_f(o[mt][3] * i1);
          }
        }
      }
    } else {
      const int slot = partial_slot(vcta, per, prefix[s]);
      float* po = p.part_o + (static_cast<int64_t>(slot) * p.n_q_heads + qh0) * 64;
      float* pml = p.part_ml + static_cast<int64_t>(slot) * p.ml_stride + qh0 * 2;
      if constexpr (FP8) {
        if constexpr (kAluV) {
#pragma unroll
          for (int j = 0; j < 4; ++j) { o[j][0] *= kCvt; o[j][1] *= kCvt; o[j][2] *= kCvt; o[j][3] *= kCvt; }
        }
        if (ok0) {
          *reinterpret_cast<float4*>(po + 8 * g) = make_float4(o[0][0], o[0][2], o[1][0], o[1][2]);
          *reinterpret_cast<float4*>(po + 8 * g + 4) = make_float4(o[2][0], o[2][2], o[3][0], o[3][2]);
        }
        if (ok1) {
          *reinterpret_cast<float4*>(po + 64 + 8 * g) = make_float4(o[0][1], o[0][3], o[1][1], o[1][3]);
          *reinterpret_cast<float4*>(po + 64 + 8 * g + 4) =
              make_float4(o[2][1], o[2][3], o[3][1], o[3][3]);
        }
      } else {
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
          if (ok0) {
            po[16 * mt + g] = o[mt][0];
            po[16 * mt + g + 8] = o[mt][2];
          }
          if (ok1) {
            po[64 + 16 * mt + g] = o[mt][1];
            po[64 + 16 * mt + g + 8] = o[mt][3];
          }
        }
      }
      if (g == 0) {
        if (ok0) { pml[0] = m0; pml[1] = lt0; }
        if (ok1) { pml[2] = m1; pml[3] = lt1; }
      }
    }
    pos = seg_end;
    s = s_next;
    if (pos < r1) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) { qa[kk][0] = qn[kk][0]; qa[kk][1] = qn[kk][1]; }
    }
  }
  if (p.defer_wait) pdl_wait();  // complete only after the kernel before this one
}

// Schedule builder: what every layer's decode launch of a step would
// otherwise recompute (clamped lengths, the block prefix, each CTA's
// stream-K range of block ids), once per step.  CTA c scans the lengths and
// writes the block ids of decode CTA c (one parallel round of table reads);
// CTA 0 also writes the header, prefix and lengths.  Bounds problems are
// flagged here, once per step; a bad block id is stored as -1.
constexpr int kSchedThreads = 128;
__global__ void __launch_bounds__(kSchedThreads) decode_schedule_kernel(
    int32_t* __restrict__ sched, const int32_t* __restrict__ tables, int64_t bt_stride,
    int max_blocks, const int32_t* __restrict__ context_lens, int B, int num_blocks, int grid,
    int rows, int* err) {
  extern __shared__ int sm_sched[];
  int* misc = sm_sched;        // scan scratch
  int* prefix = misc + 40;     // [B + 1]
  const int tid = threadIdx.x;
  const int cap_tokens = max_blocks * 16;
  const bool lead = blockIdx.x == 0;
  int32_t* ctx_out = sched + kSchedHdr + B + 1;
  for (int s = tid; s < B; s += blockDim.x) {
    int c = context_lens[s];
    if (c < 0) c = 0;
    if (c > cap_tokens) {
      if (lead) raise_flag(err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
      c = cap_tokens;
    }
    if (lead) ctx_out[s] = c;
    prefix[s] = (c + 15) >> 4;
  }
  __syncthreads();
  const int total = block_exclusive_scan(prefix, B, misc + 1);
  if (tid == 0) prefix[B] = total;
  __syncthreads();
  const int per = max((total + grid - 1) / grid, kDecMinBlocksPerCta);
  if (lead) {
    for (int s = tid; s <= B; s += blockDim.x) sched[kSchedHdr + s] = prefix[s];
    if (tid == 0) {
      sched[0] = B;
      sched[1] = total;
      sched[2] = per;
      sched[3] = grid;
      sched[4] = rows;
      sched[5] = max_blocks;
    }
  }
  int32_t* row = sched + sched_ids_offset(B) + static_cast<int64_t>(blockIdx.x) * rows;
  const int r0 = blockIdx.x * per, r1 = min(r0 + per, total);
  for (int gb = r0 + tid; gb < r1; gb += blockDim.x) {
    const int s = find_seq(prefix, B, gb);
    int id = __ldg(tables + static_cast<int64_t>(s) * bt_stride + (gb - prefix[s]));
    if (id < 0 || id >= num_blocks) {
      raise_flag(err, PKV_FLAG_BLOCK_OUT_OF_RANGE);
      id = -1;
    }
    row[gb - r0] = id;
  }
}

// Split-K merge: CTA s finishes sequence s.  If the decode kernel split it
// over CTAs c_first..c_last (stream-K ranges of `per` blocks), the partials
// (m, l, O) are merged: O = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c.
// Sequences inside one decode CTA were written by that CTA; empty sequences
// get a zero row.  Contributors are taken in chunks of kMergeChunk: all
// (m, l) of a chunk are loaded at once into shared memory, per-head weights
// are formed there, then each thread accumulates one float4 of the output
// from independent 16-byte loads, so a chunk costs two memory round trips.
// The block-count scan runs before griddepcontrol.wait and overlaps the
// decode kernel.
constexpr int kMergeThreads = 256;
constexpr int kMergeChunk = 32;
constexpr int kMergeMaxHeads = 32;

template <typename T>
__global__ void __launch_bounds__(kMergeThreads) paged_decode_merge_kernel(const DecodeParams p,
                                                                           int decode_grid) {
  __shared__ float s_m[kMergeChunk][kMergeMaxHeads];
  __shared__ float s_l[kMergeChunk][kMergeMaxHeads];
  __shared__ float s_run_m[kMergeMaxHeads], s_run_l[kMergeMaxHeads], s_scale[kMergeMaxHeads];
  __shared__ int red[2][kMergeThreads / 32];
  const int s = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cap = p.max_blocks * 16;
  int before = 0, total = 0;
  for (int i = tid; i < p.n_seqs; i += kMergeThreads) {
    const int c = min(max(p.context_lens[i], 0), cap);
    const int nb = (c + 15) >> 4;
    total += nb;
    if (i < s) before += nb;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    before += __shfl_xor_sync(0xffffffffu, before, off);
    total += __shfl_xor_sync(0xffffffffu, total, off);
  }
  if (lane == 0) { red[0][warp] = before; red[1][warp] = total; }
  __syncthreads();
  before = 0;
  total = 0;
#pragma unroll
  for (int w = 0; w < kMergeThreads / 32; ++w) { before += red[0][w]; total += red[1][w]; }
  const int nb_s = (min(max(p.context_lens[s], 0), cap) + 15) >> 4;
  const int per = max((total + decode_grid - 1) / decode_grid, kDecMinBlocksPerCta);

  pdl_wait();  // the decode grid's partials and outputs are complete and visible
  // (triggering before the wait, so that the next layer's CTAs start in SMs
  // the decode grid's tail frees, measured 2% slower)
  if (tid == 0) pdl_trigger();
  const int Hq = p.n_q_heads;
  // layer blockIdx.y of a multi-layer call (0: a single layer)
  const int64_t layer = blockIdx.y;
  T* orow = static_cast<T*>(p.out) + layer * p.out_layer_stride + static_cast<int64_t>(s) * p.out_stride;
  const float* part_o = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(p.part_o) +
                                                       layer * p.ws_layer_stride);
  const float* part_ml = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(p.part_ml) +
                                                        layer * p.ws_layer_stride);
  if (nb_s == 0) {
    for (int i = tid; i < Hq * 64; i += kMergeThreads) orow[i] = Elem<T>::from_f(0.f);
    return;
  }
  const int blk_lo = before, blk_hi = before + nb_s;
  const int c_first = blk_lo / per, c_last = (blk_hi - 1) / per;
  if (c_first == c_last) return;

  // this thread's outputs: float4 number j of the sequence row (head j / 16)
  constexpr int kOutPerThread = kMergeMaxHeads * 16 / kMergeThreads;  // 2
  float4 acc[kOutPerThread];
#pragma unroll
  for (int r = 0; r < kOutPerThread; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid < Hq) { s_run_m[tid] = -INFINITY; s_run_l[tid] = 0.f; }
  for (int c0 = c_first; c0 <= c_last; c0 += kMergeChunk) {
    const int n = min(kMergeChunk, c_last - c0 + 1);
    for (int idx = tid; idx < n * Hq; idx += kMergeThreads) {
      const int k = idx / Hq, hh = idx - k * Hq;
      const int64_t sl = partial_slot(c0 + k, per, blk_lo);
      const float2 ml = __ldcg(reinterpret_cast<const float2*>(part_ml + sl * p.ml_stride + hh * 2));
      s_m[k][hh] = ml.x;
      s_l[k][hh] = ml.y;
    }
    __syncthreads();
    if (tid < Hq) {  // running max / sum per head; s_m becomes the weight 2^(m_k - M)
      float mx = s_run_m[tid];
      for (int k = 0; k < n; ++k) mx = fmaxf(mx, s_m[k][tid]);
      const float sc = exp2f(s_run_m[tid] - mx);
      float l = s_run_l[tid] * sc;
      for (int k = 0; k < n; ++k) {
        const float w = exp2f(s_m[k][tid] - mx);
        s_m[k][tid] = w;
        l += w * s_l[k][tid];
      }
      s_run_m[tid] = mx;
      s_run_l[tid] = l;
      s_scale[tid] = sc;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kOutPerThread; ++r) {
      const int j = tid + r * kMergeThreads;
      if (j < Hq * 16) {
        const int hh = j >> 4;
        const float sc = s_scale[hh];
        float4 a = make_float4(acc[r].x * sc, acc[r].y * sc, acc[r].z * sc, acc[r].w * sc);
        for (int k0 = 0; k0 < n; k0 += 8) {
          float4 o[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (k0 + k < n) {
              const int64_t sl = partial_slot(c0 + k0 + k, per, blk_lo);
              o[k] = __ldcg(reinterpret_cast<const float4*>(part_o + sl * Hq * 64) + j);
            }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            if (k0 + k < n) {
              const float w = s_m[k0 + k][hh];
              a.x += w * o[k].x;
              a.y += w * o[k].y;
              a.z += w * o[k].z;
              a.w += w * o[k].w;
            }
          }
        }
        acc[r] = a;
      }
    }
    __syncthreads();  // s_m / s_scale are rewritten by the next chunk
  }
#pragma unroll
  for (int r = 0; r < kOutPerThread; ++r) {
    const int j = tid + r * kMergeThreads;
    if (j < Hq * 16) {
      const float inv = 1.f / s_run_l[j >> 4];
      uint2 v;
      v.x = pack2<T>(acc[r].x * inv, acc[r].y * inv);
      v.y = pack2<T>(acc[r].z * inv, acc[r].w * inv);
      *reinterpret_cast<uint2*>(orow + 4 * j) = v;
    }
  }
}

// pipelines (virtual CTAs) per CTA: one CTA per SM holds as many as 5 CTAs
// of one pipeline would (the register limit) for two KV heads; other head
// counts keep one pipeline per CTA
#ifndef PKV_DEC_PIPES
#define PKV_DEC_PIPES 5
#endif
constexpr int pipes_for(int nkv) { return nkv == 2 ? PKV_DEC_PIPES : 1; }

size_t decode_smem_bytes(int nkv, int n_seqs, bool fp8) {
  const size_t stage = fp8 ? 2 * nkv * kDecTile8 + 2 * 16 * nkv * 4 : 2 * nkv * kDecTile;
  const int stages = fp8 ? dec_stages<true>() : dec_stages<false>();
  return 1024 +
         static_cast<size_t>(pipes_for(nkv)) *
             (static_cast<size_t>(stages) * stage + 2 * stages * sizeof(uint64_t)) +
         40 * sizeof(int) + (2 * static_cast<size_t>(n_seqs) + 1) * sizeof(int);
}

namespace {
struct OccKey {
  int dev, kind, smem, threads;
  bool operator==(const OccKey& o) const {
    return dev == o.dev && kind == o.kind && smem == o.smem && threads == o.threads;
  }
};
struct OccHash {
  size_t operator()(const OccKey& k) const {
    return (static_cast<size_t>(k.dev) * 131 + k.kind) * 1000003u + k.smem * 7 + k.threads;
  }
};
std::mutex g_occ_mu;
std::unordered_map<OccKey, int, OccHash> g_occ;

using DecodeKernel = void (*)(const CUtensorMap, const CUtensorMap, const DecodeParams);

template <bool FP8>
DecodeKernel pick_kernel_t(int dtype, int nkv) {
  if (dtype == PKV_DTYPE_F16)
    return nkv == 1   ? paged_decode_kernel<__half, 1, FP8, pipes_for(1)>
           : nkv == 2 ? paged_decode_kernel<__half, 2, FP8, pipes_for(2)>
                      : paged_decode_kernel<__half, 4, FP8, pipes_for(4)>;
  return nkv == 1   ? paged_decode_kernel<__nv_bfloat16, 1, FP8, pipes_for(1)>
         : nkv == 2 ? paged_decode_kernel<__nv_bfloat16, 2, FP8, pipes_for(2)>
                    : paged_decode_kernel<__nv_bfloat16, 4, FP8, pipes_for(4)>;
}
DecodeKernel pick_kernel(int dtype, int nkv, bool fp8) {
  return fp8 ? pick_kernel_t<true>(dtype, nkv) : pick_kernel_t<false>(dtype, nkv);
}
}  // namespace

// the persistent grid of the decode kernel for this shape, in virtual CTAs
// (pipelines; cached occupancy); the launch has grid / pipes_for(nkv) CTAs
cudaError_t decode_grid(int dtype, int nkv, bool fp8, int n_seqs, int* grid_out) {
  const int pipes = pipes_for(nkv);
  const int threads = 32 * (nkv + 1) * pipes;
  const size_t smem = decode_smem_bytes(nkv, n_seqs, fp8);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  DecodeKernel kern = pick_kernel(dtype, nkv, fp8);
  const int kind = dtype * 8 + nkv + (fp8 ? 64 : 0);
  int grid = 0;
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    const OccKey key{dev, kind, static_cast<int>(smem), threads};
    auto it = g_occ.find(key);
    if (it == g_occ.end()) {
      // one opt-in size per (device, kernel): the largest any call can need
      const OccKey attr_key{dev, kind, -1, 0};
      if (g_occ.find(attr_key) == g_occ.end()) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(decode_smem_bytes(nkv, kDecMaxSeqs, fp8)));
        if (e != cudaSuccess) return e;
        g_occ.emplace(attr_key, 0);
      }
      int per_sm = 0, sms = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
      if (e != cudaSuccess) return e;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      it = g_occ.emplace(key, pipes * std::max(1, std::min(kDecMaxCtas / pipes, per_sm * sms))).first;
    }
    grid = it->second;
  }
  *grid_out = grid;
  return cudaSuccess;
}

namespace {
// The decode kernel reads its schedule before griddepcontrol.wait, so a decode
// launch may overlap its predecessor only if the schedule is known to be
// complete: a decode launch has already read it since its last build.  This
// table maps a schedule to that fact.  A schedule that was just built, or one
// the table does not know (never seen, or forgotten when the table was
// cleared), gets a stream-ordered launch; clearing the table therefore costs
// at most one overlap per schedule and never lets a launch read a schedule
// that is still being written.
constexpr size_t kSchedTableMax = 4096;
std::mutex g_sched_mu;
std::unordered_map<const void*, bool> g_sched_read;

void sched_table_set(const void* schedule, bool read) {
  if (g_sched_read.size() >= kSchedTableMax && g_sched_read.find(schedule) == g_sched_read.end())
    g_sched_read.clear();
  g_sched_read[schedule] = read;
}
}  // namespace

cudaError_t launch_decode_schedule(void* schedule, const AttnArgs& a, cudaStream_t stream) {
  const bool fp8 = a.k_scale != nullptr;
  int grid = 0;
  cudaError_t e = decode_grid(a.dtype, a.n_kv_heads, fp8, a.n_seqs, &grid);
  if (e != cudaSuccess) return e;
  const int rows = sched_rows_for(a.n_seqs, a.max_blocks, grid);
  const size_t smem = (40 + static_cast<size_t>(a.n_seqs) + 1) * sizeof(int);
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(decode_schedule_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  decode_schedule_kernel<<<grid, kSchedThreads, smem, stream>>>(
      static_cast<int32_t*>(schedule), a.block_tables, a.bt_stride, a.max_blocks, a.context_lens,
      a.n_seqs, a.num_blocks, grid, rows, a.err);
  e = cudaGetLastError();
  if (e == cudaSuccess) {
    std::lock_guard<std::mutex> lk(g_sched_mu);
    sched_table_set(schedule, false);
  }
  return e;
}

cudaError_t launch_decode_fast(const AttnArgs& a, const CUtensorMap* kmap, const CUtensorMap* vmap,
                               void* workspace, cudaStream_t stream) {
  if (a.n_seqs == 0) return cudaSuccess;
  const int nkv = a.n_kv_heads;
  const int threads = 32 * (nkv + 1) * pipes_for(nkv);
  const bool fp8 = a.k_scale != nullptr;
  const size_t smem = decode_smem_bytes(nkv, a.n_seqs, fp8);
  DecodeKernel kern = pick_kernel(a.dtype, nkv, fp8);
  int grid = 0;
  cudaError_t e = decode_grid(a.dtype, nkv, fp8, a.n_seqs, &grid);
  if (e != cudaSuccess) return e;
  bool ordered = false;  // no programmatic overlap unless the schedule is known complete
  if (a.schedule != nullptr) {
    std::lock_guard<std::mutex> lk(g_sched_mu);
    auto it = g_sched_read.find(a.schedule);
    ordered = it == g_sched_read.end() || !it->second;
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
  p.ml_stride = (2 * a.n_q_heads + 3) & ~3;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float*>(ws + parts_o);
  p.err = a.err;
  p.k_new = static_cast<const uint8_t*>(a.k_new);
  p.v_new = static_cast<const uint8_t*>(a.v_new);
  p.k_new_stride_b = a.k_new_stride * 2;
  p.v_new_stride_b = a.v_new_stride * 2;
  p.k_pool = static_cast<uint8_t*>(const_cast<void*>(a.k_pool));
  p.v_pool = static_cast<uint8_t*>(const_cast<void*>(a.v_pool));
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  p.sched = static_cast<const int32_t*>(a.schedule);
  p.sched_rows = a.schedule != nullptr ? sched_rows_for(a.n_seqs, a.max_blocks, grid) : 0;
  p.input_ready = a.input_ready;
  p.defer_wait = a.chain != nullptr ? a.chain->defer_wait : 0;
  p.late_trigger = a.chain != nullptr && !a.chain->defer_wait;
  p.out_layer_stride = 0;
  p.ws_layer_stride = 0;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid / pipes_for(nkv));
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ordered ? 0 : 1;
  e = cudaLaunchKernelEx(&cfg, kern, *kmap, *vmap, p);
  if (e != cudaSuccess) return e;
  if (a.schedule != nullptr) {  // read by a launch that is now queued behind its build
    std::lock_guard<std::mutex> lk(g_sched_mu);
    sched_table_set(a.schedule, true);
  }

  if (a.chain != nullptr && !a.chain->merge) return cudaSuccess;  // a later launch merges
  if (a.chain != nullptr) {  // the merge of every layer of the call
    const LayerChain& ch = *a.chain;
    uint8_t* ws0 = static_cast<uint8_t*>(ch.ws0);
    p.out = ch.out0;
    p.part_o = reinterpret_cast<float*>(ws0);
    p.part_ml = reinterpret_cast<float*>(ws0 + parts_o);
    p.out_layer_stride = ch.out_layer_stride;
    p.ws_layer_stride = ch.ws_layer_stride;
  }
  cudaLaunchConfig_t mcfg = cfg;
  mcfg.numAttrs = 1;
  mcfg.gridDim = dim3(a.n_seqs, a.chain != nullptr ? a.chain->n_layers : 1);
  mcfg.blockDim = dim3(kMergeThreads);
  mcfg.dynamicSmemBytes = 0;
  if (a.dtype == PKV_DTYPE_F16)
    return cudaLaunchKernelEx(&mcfg, paged_decode_merge_kernel<__half>, p, grid);
  return cudaLaunchKernelEx(&mcfg, paged_decode_merge_kernel<__nv_bfloat16>, p, grid);
}

}  // namespace pkv
