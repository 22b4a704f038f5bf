// pkv_prefill.cu -- paged chunked-prefill attention on the 5th-generation tensor
// cores (tcgen05 + tensor memory), fp16 / bf16 KV, head_dim 64, 16-token blocks.
//
// Replaces the reference's per-sequence gather + _attention for num_new > 1
// (mini_engine/paged/block_manager.py:136-141, mini_engine/model/qwen2.py:98-128):
// query i of sequence s attends to keys 0 .. num_prior[s] + i, with the prefix
// blocks (shared radix-cache blocks included) read in place through the
// block table.
//
// One CTA per (sequence, query head, pair of 128-query tiles A and B); the two
// tiles share every K/V tile the CTA loads.  12 warps (three warpgroups):
//  * warps 0-3 / 4-7 (softmax of tile A / tile B): thread r of a group owns
//    query row r of its tile.  It reads its row of S = Q K^T from TMEM
//    (tcgen05.ld), applies the causal mask and an online softmax in the exp2
//    domain, writes its row of P (fp16/bf16 pairs) back into TMEM
//    (tcgen05.st), and at the end reads O from TMEM, normalises and stores it.
//    O is rescaled in TMEM only when the running maximum grows by more than 8
//    (2^8 bounds P), so rescaling is rare.  The two groups run side by side
//    (two warps per SM sub-partition), so one group's exponentials overlap
//    the other's tensor-memory traffic and barrier waits.
//  * warp 8 (producer): TMA tensor loads of the two Q tiles (once) and, per
//    key tile of 128 keys (8 blocks), the K and V blocks into a 4-stage ring;
//    blocks past the visible keys are fetched from an out-of-range coordinate
//    and arrive as zeros.
//  * warps 9 and 10 (MMA; fp8: warp 9 alone): warp 9 allocates all 512 TMEM
//    columns (S_A, S_B: 128 fp32 each; O_A, O_B: 64 fp32 each; P_A, P_B: 64
//    columns of fp16/bf16 pairs each).  Warp 9 issues tile A's MMAs and warp
//    10 tile B's, so neither tile's next S or PV waits on the other tile's
//    softmax (2% over one issuer for both); one elected lane of each issues
//    tcgen05.mma kind::f16 (M=128):
//    S_x = Q_x K_j^T (N=128, K=64, both K-major, from shared memory) and
//    O_x += P_x V_j (N=64, K=128; A = P_x from tensor memory, B = V the
//    MN-major shared operand), committing to mbarriers.  S_x of key tile j+1
//    is issued as soon as the softmax holds S_x of tile j in registers, so
//    QK^T overlaps the exponentials.  Keeping P in tensor memory halves the
//    shared-memory traffic of a key tile (no P stores, no P operand reads).
// Tile B of a CTA may need one key tile more than tile A (its last rows see
// 128 more keys); that tile is loaded once and only B computes on it.
//
// CTA order.  Work items differ in length by up to the whole context, and one
// CTA fills an SM, so the grid is mapped longest-first: blockIdx.x enumerates
// sequences by decreasing (prior + new) length, then the later query pair of a
// sequence, then the head.  The hardware dispatches CTAs in blockIdx order as
// SMs free up, which makes this a longest-processing-time list schedule.  The
// rank is computed by every CTA from num_prior / query_start_loc (up to
// kPfOrderMaxSeqs sequences; natural order beyond).
//
// Registers.  The 384 threads launch with 168 registers each (64,512 in all).
// The third warpgroup (producer, MMA, two idle warps) gives registers back with
// setmaxnreg.dec to 56 and the two softmax warpgroups raise theirs to 224:
// 128 x 56 + 256 x 224 = 64,512, the launch total.  The host checks the compiled
// register count against that sum before the first launch (a split above the
// launch total would leave setmaxnreg.inc waiting).
//
// Every wait is bounded; on a timeout the kernel flags PKV_FLAG_PIPELINE_TIMEOUT,
// stops waiting and still frees its tensor memory.
#include <float.h>

#include <mutex>
#include <type_traits>

#include "pkv_common.cuh"
#include "pkv_internal.h"

namespace pkv {

constexpr int kPfM = 128;                 // query rows per tile
constexpr int kPfPair = 2 * kPfM;         // query rows per CTA (tiles A and B)
constexpr int kPfN = 128;                 // keys per tile (8 blocks of 16)
#ifndef PKV_PF_STAGES
#define PKV_PF_STAGES 4
#endif
constexpr int kPfStages = PKV_PF_STAGES;  // K/V ring depth
constexpr int kPfTile = 128 * 64 * 2;     // 16 KB: 128 rows x 64 dims x 2 bytes
constexpr int kPfThreads = 384;
constexpr int kPfRegsSoftmax = 224;       // per thread, warpgroups 0 and 1
constexpr int kPfRegsOther = 56;          // per thread, warpgroup 2
constexpr int kPfRegSplit = 256 * kPfRegsSoftmax + 128 * kPfRegsOther;
constexpr int kPfProducerWarp = 8;
constexpr int kPfMmaWarp = 9;
constexpr uint32_t kPfTmemCols = 512;
constexpr int kPfOrderMaxSeqs = 64;
#ifndef PKV_PF_POLY_EVERY
#define PKV_PF_POLY_EVERY 3
#endif
// one key pair in kPfPolyEvery takes the FMA-pipe exp2 (0: all on the MUFU);
// with the paired fp32 instructions a pair's polynomial costs about a dozen
// issue slots, and one pair in three measured best (1/2: 610, 1/3: 624,
// 1/4: 622, 1/5: 611, 1/8: 598 TFLOP/s over the config-4 step)
constexpr int kPfPolyEvery = PKV_PF_POLY_EVERY;

// tensor-memory columns: S_A, S_B (fp32), O_A, O_B (fp32), P_A, P_B (fp16/bf16 pairs)
constexpr uint32_t kColS = 0, kColO = 256, kColP = 384;

// shared-memory offsets from the 1024-byte aligned base
constexpr int kOffQ = 0;                               // Q_A, Q_B
constexpr int kOffK = kOffQ + 2 * kPfTile;
constexpr int kOffV = kOffK + kPfStages * kPfTile;
constexpr int kOffBar = kOffV + kPfStages * kPfTile;
constexpr int kNumBars = 1 + 2 * kPfStages + 4 * 2 + 2 * 2;
constexpr int kOffSched = kOffBar + kNumBars * 8;      // tmem slot, work item, length keys
constexpr int kSchedInts = 4 + kPfOrderMaxSeqs;
constexpr int kPfSmemBytes = 1024 + kOffSched + kSchedInts * 4;
static_assert(kPfSmemBytes <= 232448, "prefill ring does not fit the 227 KB of shared memory per CTA");
// fp8 pools: a 2-stage ring of the raw e4m3 key tiles (128 keys x 64 bytes for
// K and for V) and their rows' fp32 scales (8 blocks x 16 rows x up to
// kPf8MaxKvHeads heads), after the 16-bit ring, 1024-byte aligned
constexpr int kPf8Stages = 2;
constexpr int kPf8MaxKvHeads = 4;
constexpr int kPf8Tile = 128 * 64;                     // 8 KB of e4m3
constexpr int kPf8Scales = 8 * 16 * kPf8MaxKvHeads * 4;  // one tile's scales, K or V
constexpr int kPf8Stage = 2 * kPf8Tile + 2 * kPf8Scales;
constexpr int kOffS8 = (kOffSched + kSchedInts * 4 + 1023) / 1024 * 1024;
constexpr int kPfSmemBytesFp8 = 1024 + kOffS8 + kPf8Stages * kPf8Stage;
static_assert(kPfSmemBytesFp8 <= 232448, "fp8 staging does not fit the 227 KB of shared memory per CTA");
constexpr int kPfConvWarp0 = 10;  // warps 10 and 11 convert the fp8 tiles

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
  int n_seqs;
  int n_q_heads;
  int n_pairs;         // query pairs per sequence in the grid: ceil(max_query_len / 256)
  int order_by_length;
  int group;
  float scale_log2;
  int* err;
  // fp8 pools: fp32 scale per (slot, KV head)
  const float* k_scale;
  const float* v_scale;
  int n_kv_heads;
};

template <typename T, bool FP8>
__global__ void __launch_bounds__(kPfThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kPfStages;
  uint64_t* s_full = kv_empty + kPfStages;  // [tile]: S_x of the current key tile is in TMEM
  uint64_t* s_empty = s_full + 2;           // [tile]: the softmax holds S_x in registers
  uint64_t* p_full = s_empty + 2;           // [tile]: P_x is in tensor memory
  uint64_t* o_done = p_full + 2;            // [tile]: O_x += P_x V has completed
  uint64_t* s8_full = o_done + 2;           // fp8: the raw tiles and scales of a stage landed
  uint64_t* s8_empty = s8_full + kPf8Stages;  // fp8: the converters are done with a stage
  int* sched = reinterpret_cast<int*>(base + kOffSched);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sched);
  const uint32_t sbase = smem_u32(base);

  // ---- work item of this CTA (warp 0), barriers (warp 1), TMEM (MMA warp)
  if (warp == 0) {
    const int per_seq = p.n_pairs * p.n_q_heads;
    const int rho = static_cast<int>(blockIdx.x) / per_seq;
    const int rem = static_cast<int>(blockIdx.x) - rho * per_seq;
    if (lane == 0) {
      sched[1] = rho;
      sched[2] = p.n_pairs - 1 - rem / p.n_q_heads;
      sched[3] = rem % p.n_q_heads;
    }
    if (p.order_by_length) {
      // rank of sequence t: how many sequences are longer, ties by index
      int* keys = sched + 4;
      for (int t = lane; t < p.n_seqs; t += 32)
        keys[t] = max(p.num_prior[t], 0) + (p.qsl[t + 1] - p.qsl[t]);
      __syncwarp();
      for (int t = lane; t < p.n_seqs; t += 32) {
        const int kt = keys[t];
        int rank = 0;
        for (int u = 0; u < p.n_seqs; ++u) {
          const int ku = keys[u];
          rank += (ku > kt) || (ku == kt && u < t);
        }
        if (rank == rho) sched[1] = t;  // ranks are a permutation: one writer
      }
    }
  } else if (warp == 1 && lane == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kPfStages; ++i) {
      // fp8: the 16-bit tiles are written by the two converter warps
      mbar_init(&kv_full[i], FP8 ? 2 : 1);
      // 16-bit: both MMA warps (one per query tile) release each stage
      mbar_init(&kv_empty[i], FP8 ? 1 : 2);
    }
    for (int i = 0; i < kPf8Stages; ++i) {
      mbar_init(&s8_full[i], 1);
      mbar_init(&s8_empty[i], 2);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    fence_barrier_init();
  } else if (warp == kPfMmaWarp) {
    tmem_alloc(tmem_slot, kPfTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Launched with programmatic serialization: the set-up above (work item,
  // barriers, tensor memory; it reads only the step's metadata, which no
  // preceding kernel of the chain writes) overlaps the kernel before this
  // one.  Q, the pools (the append before this kernel writes them) and out
  // are touched only after the wait.  The trigger lets the next kernel
  // launch once every CTA of this grid has started.
  if (tid == 0) pdl_trigger();
  pdl_wait();
  const uint32_t tbase = *tmem_slot;
  const int s = sched[1], qp = sched[2], h = sched[3];

  const int q_begin = p.qsl[s];
  const int n_new = p.qsl[s + 1] - q_begin;
  const int q0 = qp * kPfPair;
  bool skip = false;
  if (qp == p.n_pairs - 1 && h == 0 && n_new > p.n_pairs * kPfPair && tid == 0)
    raise_flag(p.err, PKV_FLAG_BAD_QUERY_LAYOUT);  // max_query_len below a chunk length
  if (q_begin < 0 || n_new < 0 || q_begin + n_new > p.n_tokens) {
    if (qp == 0 && h == 0 && tid == 0) raise_flag(p.err, PKV_FLAG_BAD_QUERY_LAYOUT);
    skip = true;
  }
  if (skip || n_new == 0 || q0 >= n_new) {  // uniform over the CTA
    if (warp == kPfMmaWarp) tmem_dealloc(tbase, kPfTmemCols);
    return;
  }
  const int prior = max(p.num_prior[s], 0);
  const int cap = p.max_blocks * 16;
  // tile x covers queries q0 + 128 x ...; kv[x] keys are visible to its last row
  int rows[2], kv[2], nt[2];
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    rows[x] = min(max(n_new - (q0 + x * kPfM), 0), kPfM);
    kv[x] = rows[x] > 0 ? prior + q0 + x * kPfM + rows[x] : 0;
    if (kv[x] > cap) {
      if (tid == 0) raise_flag(p.err, PKV_FLAG_CONTEXT_EXCEEDS_TABLE);
      kv[x] = cap;
    }
    nt[x] = (kv[x] + kPfN - 1) / kPfN;
  }
  const int n_kv_tiles = max(nt[0], nt[1]);
  const int nb_needed = (max(kv[0], kv[1]) + 15) >> 4;
  const int g = h / p.group;

  if (warp >= 8) {
  // third warpgroup: producer, MMA issuer, two idle warps
  setmaxnreg_dec<kPfRegsOther>();
  if (warp == kPfProducerWarp) {
    // ======================= producer =======================
    // warp-converged; one elected lane issues the TMA loads
    if (elect_one()) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      mbar_arrive_expect_tx(q_full, rows[1] > 0 ? 2 * kPfTile : kPfTile);
      tma_load_3d(base + kOffQ, &qmap, q_full, 0, h, q_begin + q0);
      if (rows[1] > 0) tma_load_3d(base + kOffQ + kPfTile, &qmap, q_full, 0, h, q_begin + q0 + kPfM);
    }
    __syncwarp();
    for (int j = 0; j < n_kv_tiles; ++j) {
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
      if constexpr (FP8) {
        // raw e4m3 tiles and their rows' scales into the staging ring; the
        // converter warps turn them into the 16-bit ring's tiles
        const int s8 = j % kPf8Stages;
        if (!__all_sync(0xffffffffu, mbar_wait(&s8_empty[s8], ((j / kPf8Stages) & 1) ^ 1))) {
          if (lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
          break;
        }
        const int nvalid = min(max(nb_needed - j * 8, 0), 8);  // blocks with keys: a prefix
        const int sbytes = 16 * p.n_kv_heads * 4;
        if (elect_one()) {
          uint8_t* stg = base + kOffS8 + s8 * kPf8Stage;
          mbar_arrive_expect_tx(&s8_full[s8], 2 * kPf8Tile + 2 * nvalid * sbytes);
#pragma unroll
          for (int b = 0; b < 8; ++b) {
            tma_load_3d(stg + b * 1024, &kmap, &s8_full[s8], 0, g, toks[b]);
            tma_load_3d(stg + kPf8Tile + b * 1024, &vmap, &s8_full[s8], 0, g, toks[b]);
          }
          for (int b = 0; b < nvalid; ++b) {
            const int64_t so = static_cast<int64_t>(toks[b]) * p.n_kv_heads;  // row (block*16) x heads
            bulk_load(stg + 2 * kPf8Tile + b * sbytes, p.k_scale + so, sbytes, &s8_full[s8]);
            bulk_load(stg + 2 * kPf8Tile + kPf8Scales + b * sbytes, p.v_scale + so, sbytes, &s8_full[s8]);
          }
        }
        __syncwarp();
        continue;
      }
      const int st = j % kPfStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&kv_empty[st], ((j / kPfStages) & 1) ^ 1))) {
        if (lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
        break;
      }
      if (elect_one()) {
        mbar_arrive_expect_tx(&kv_full[st], 2 * kPfTile);
        uint8_t* kd = base + kOffK + st * kPfTile;
        uint8_t* vd = base + kOffV + st * kPfTile;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          tma_load_3d(kd + b * 2048, &kmap, &kv_full[st], 0, g, toks[b]);
          tma_load_3d(vd + b * 2048, &vmap, &kv_full[st], 0, g, toks[b]);
        }
      }
      __syncwarp();
    }
  } else if (warp == kPfMmaWarp || (!FP8 && warp == kPfMmaWarp + 1)) {
    // ======================= MMA issuers =======================
    // The whole warp runs the loop, so descriptors and tensor-memory
    // addresses are warp-uniform values; one elected lane (the same lane every
    // time) issues every tcgen05.mma and tcgen05.commit (a commit tracks the
    // operations of the thread that issues it).
    constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t idesc_s = mma_idesc_f16(fmt, 0, 0, kPfN, kPfM);
    constexpr uint32_t idesc_o = mma_idesc_f16(fmt, 0, 1, 64, kPfM);
    auto wait_all = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity));
    };
    auto issue_qk = [&](int x, int j) {
      const uint32_t qa = sbase + kOffQ + x * kPfTile;
      const uint32_t ka = sbase + kOffK + (j % kPfStages) * kPfTile;
      uint64_t ad[4], bd[4];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        ad[kk] = smem_desc(qa + kk * 32, 16, 1024);
        bd[kk] = smem_desc(ka + kk * 32, 16, 1024);
      }
      if (elect_one()) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_f16(tbase + kColS + x * 128, ad[kk], bd[kk], idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(&s_full[x]);
      }
      __syncwarp();
    };
    auto issue_pv = [&](int x, int j) {
      // A = P_x from tensor memory: 16 keys (8 columns) per instruction
      const uint32_t va = sbase + kOffV + (j % kPfStages) * kPfTile;
      uint64_t bd[8];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) bd[kk] = smem_desc(va + kk * 2048, 16, 1024);
      if (elect_one()) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_f16_ts(tbase + kColO + x * 64, tbase + kColP + x * 64 + kk * 8, bd[kk], idesc_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&o_done[x]);
      }
      __syncwarp();
    };
    // 16-bit: warp 9 issues tile A's MMAs and warp 10 tile B's, so neither
    // tile's next S or PV waits on the other tile's softmax; fp8 (warps 10
    // and 11 convert): warp 9 issues both.  Each warp waits for every key
    // tile and releases every stage, including tiles its query tile does not
    // reach, so a release always follows that stage's load.
    const int xs = FP8 ? -1 : warp - kPfMmaWarp;  // the query tile this warp serves (-1: both)
    auto serves = [&](int x) { return xs < 0 || x == xs; };
    bool dead = !wait_all(q_full, 0);
    if (!dead && !wait_all(&kv_full[0], 0)) dead = true;
    if (!dead) {
      if (serves(0) && nt[0] > 0) issue_qk(0, 0);
      if (serves(1) && nt[1] > 0) issue_qk(1, 0);
    }
    for (int j = 0; j < n_kv_tiles && !dead; ++j) {
      // S of key tile j+1 once the softmax has read S of tile j
      if (j + 1 < n_kv_tiles && !wait_all(&kv_full[(j + 1) % kPfStages], ((j + 1) / kPfStages) & 1)) {
        dead = true;
        break;
      }
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (!serves(x) || j + 1 >= nt[x]) continue;
        if (!wait_all(&s_empty[x], j & 1)) {
          dead = true;
          break;
        }
        issue_qk(x, j + 1);
      }
      if (dead) break;
      // O_x += P_x V_j once the softmax has written P_x
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (!serves(x) || j >= nt[x]) continue;
        if (!wait_all(&p_full[x], j & 1)) {
          dead = true;
          break;
        }
        issue_pv(x, j);
      }
      if (dead) break;
      if (elect_one()) tc_commit(&kv_empty[j % kPfStages]);
      __syncwarp();
    }
    if (dead && lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
  } else if (FP8 && warp >= kPfConvWarp0) {
    // ======================= fp8 converters (warps 10, 11) =======================
    // Key tile j: wait for its raw stage and for the 16-bit ring stage to be
    // free, then each of the 64 threads converts 4 of the tile's 256 rows (128
    // of K, 128 of V): 64 e4m3 bytes -> 64 fp16 values x the row's scale,
    // stored with the 128-byte swizzle the MMA descriptors read (16-byte chunk
    // c of row r at c ^ (r & 7)).  The conversion moves the e4m3 fields into
    // f16 position on the integer pipes (the value x 2^-8, exact), widens to
    // fp32 and multiplies by (scale x 2^8): one rounding of the product, as
    // the 16-bit scratch pass computes it (no transcendental-pipe work: that
    // pipe bounds the softmax).  Rows past the CTA's last visible key are
    // written as zeros (an unused slot may hold any bytes).
    const int u = (warp - kPfConvWarp0) * 32 + lane;
    const int kv_max = max(kv[0], kv[1]);
    const int hkv = p.n_kv_heads;
    bool dead = false;
    for (int j = 0; j < n_kv_tiles; ++j) {
      const int s8 = j % kPf8Stages, st = j % kPfStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&s8_full[s8], (j / kPf8Stages) & 1)) ||
          !__all_sync(0xffffffffu, mbar_wait(&kv_empty[st], ((j / kPfStages) & 1) ^ 1))) {
        dead = true;
        break;
      }
      const uint8_t* stg = base + kOffS8 + s8 * kPf8Stage;
      for (int rr = u; rr < 2 * kPfN; rr += 64) {
        const bool isv = rr >= kPfN;
        const int r = rr & (kPfN - 1);
        const uint8_t* src = stg + (isv ? kPf8Tile : 0) + r * 64;
        uint8_t* dst = base + (isv ? kOffV : kOffK) + st * kPfTile + r * 128;
        const int sw = r & 7;
        if (j * kPfN + r < kv_max) {
          const float* scl = reinterpret_cast<const float*>(stg + 2 * kPf8Tile + (isv ? kPf8Scales : 0));
          // (e4m3 x 2^-8) x (scale x 2^8): the 2^8 factors are exact, so the
          // fp32 product is e4m3 x scale rounded once, then once to fp16
          const float sc2 = scl[(r >> 4) * 16 * hkv + (r & 15) * hkv + g] * 256.f;
#pragma unroll
          for (int c16 = 0; c16 < 4; ++c16) {
            const uint4 w = *reinterpret_cast<const uint4*>(src + c16 * 16);
            const uint32_t in[4] = {w.x, w.y, w.z, w.w};
            uint32_t o[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // even bytes (0, 2) and odd bytes (1, 3) of the word, as f16 pairs
              const uint32_t ev = e4m3_even_h2(in[k]), od = e4m3_odd_h2(in[k]);
              const float2 fe = __half22float2(*reinterpret_cast<const __half2*>(&ev));
              const float2 fo = __half22float2(*reinterpret_cast<const __half2*>(&od));
              o[2 * k] = pack2<__half>(fe.x * sc2, fo.x * sc2);      // values 4k, 4k + 1
              o[2 * k + 1] = pack2<__half>(fe.y * sc2, fo.y * sc2);  // values 4k + 2, 4k + 3
            }
            *reinterpret_cast<uint4*>(dst + (((2 * c16) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(dst + (((2 * c16 + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        } else {
          const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dst + (c << 4)) = z;
        }
      }
      fence_proxy_async_smem();  // the generic-proxy tile writes, before the tensor core reads them
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&kv_full[st]);
        mbar_arrive(&s8_empty[s8]);
      }
    }
    if (dead && lane == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
  }
  } else {
    setmaxnreg_inc<kPfRegsSoftmax>();
    // ======================= softmax / epilogue (thread = query row) =======================
    const int x = warp >> 2;
    const int r = tid & 127;
    const int ntx = x ? nt[1] : nt[0];  // selects keep the per-tile arrays in registers
    const bool row_valid = r < (x ? rows[1] : rows[0]);
    const int lim = row_valid ? min(prior + q0 + x * kPfM + r + 1, x ? kv[1] : kv[0]) : 0;  // keys [0, lim)
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tbase + kColS + x * 128 + lane_off;
    const uint32_t t_o = tbase + kColO + x * 64 + lane_off;
    const uint32_t t_p = tbase + kColP + x * 64 + lane_off;
    const float sl2 = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool dead = false;
    for (int j = 0; j < ntx; ++j) {
      if (!dead && !mbar_wait(&s_full[x], j & 1)) dead = true;
      __syncwarp();  // tcgen05.ld is warp-collective
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) tmem_ld32(t_s + c4 * 32, sr[c4]);
      tmem_wait_ld_regs(sr[0]);
      reg_after_wait(sr[1]);
      reg_after_wait(sr[2]);
      reg_after_wait(sr[3]);
      tc_fence_before();
      mbar_arrive(&s_empty[x]);

      // keys at or past this row's causal limit become -inf (exp2 -> 0)
      const int kbase = j * kPfN;
      if (kbase + kPfN > lim) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (kbase + c >= lim) sr[c >> 5][c & 31] = __float_as_uint(-INFINITY);
      }
      // row max on raw scores (scale > 0 is checked on the host): eight
      // independent chains of three-input max
      float m8[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) m8[q] = fmaxf(__uint_as_float(sr[0][q]), __uint_as_float(sr[0][q + 8]));
#pragma unroll
      for (int c = 16; c < 128; c += 16) {  // columns c + q and c + 8 + q
#pragma unroll
        for (int q = 0; q < 8; ++q)
          m8[q] = fmax3(m8[q], __uint_as_float(sr[c >> 5][(c & 31) + q]),
                        __uint_as_float(sr[(c + 8) >> 5][((c + 8) & 31) + q]));
      }
      const float mt = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]),
                             fmaxf(m8[6], m8[7])) * sl2;
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
      // P in two halves of 64 keys: the first half covers the wait for the
      // PV of tile j-1 (which last read P_x and last wrote O_x)
      // key pairs through the paired fp32 instructions of sm_100 (one
      // issue slot per pair for the scale-and-shift and for the row sum)
      float2 ls[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 sl2v = make_float2(sl2, sl2), nmv = make_float2(nm, nm);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int c2 = half * 32 + i, c = 2 * c2;
          const float2 xs = __ffma2_rn(make_float2(__uint_as_float(sr[c >> 5][c & 31]),
                                                   __uint_as_float(sr[(c + 1) >> 5][(c + 1) & 31])),
                                       sl2v, nmv);
          const bool poly = kPfPolyEvery > 0 && (c2 % (kPfPolyEvery > 0 ? kPfPolyEvery : 1)) == kPfPolyEvery - 1;
          const float2 pp = poly ? exp2_poly3x2(xs) : make_float2(ex2_approx(xs.x), ex2_approx(xs.y));
          ls[i & 1] = __fadd2_rn(ls[i & 1], pp);
          pk[i] = pack2<T>(pp.x, pp.y);
        }
        if (half == 0) {
          if (j >= 1 && !dead && !mbar_wait(&o_done[x], (j - 1) & 1)) dead = true;
          __syncwarp();
          tc_fence_after();
          if (rescale) {
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {
              uint32_t orr[32];
              tmem_ld32(t_o + c2 * 32, orr);
              tmem_wait_ld_regs(orr);
#pragma unroll
              for (int c = 0; c < 32; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * factor);
              tmem_st32(t_o + c2 * 32, orr);
            }
          }
        }
        // row r of P: 64 columns of packed (even key, odd key) pairs
        tmem_st32(t_p + half * 32, pk);
      }
      l += (ls[0].x + ls[1].x) + (ls[0].y + ls[1].y);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    // ---- epilogue: O / l -> out
    uint32_t o0[32], o1[32];
    if (ntx > 0) {
      if (!dead && !mbar_wait(&o_done[x], (ntx - 1) & 1)) dead = true;
      __syncwarp();
      tc_fence_after();
      tmem_ld32(t_o, o0);
      tmem_ld32(t_o + 32, o1);
      tmem_wait_ld_regs(o0);
      reg_after_wait(o1);
    }
    if (dead && r == 0) raise_flag(p.err, PKV_FLAG_PIPELINE_TIMEOUT);
    if (row_valid) {
      // no visible key (a table of zero blocks): the row is zeros
      const float inv = (ntx > 0 && l > 0.f) ? 1.f / l : 0.f;
      T* orow = static_cast<T*>(p.out) + static_cast<int64_t>(q_begin + q0 + x * kPfM + r) * p.out_stride +
                static_cast<int64_t>(h) * 64;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        const uint32_t* src = c8 < 4 ? o0 + c8 * 8 : o1 + (c8 - 4) * 8;
        float f[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = inv == 0.f ? 0.f : __uint_as_float(src[i]) * inv;
        uint4 v;
        v.x = pack2<T>(f[0], f[1]);
        v.y = pack2<T>(f[2], f[3]);
        v.z = pack2<T>(f[4], f[5]);
        v.w = pack2<T>(f[6], f[7]);
        *reinterpret_cast<uint4*>(orow + c8 * 8) = v;
      }
    }
  }
  // ---- teardown: every tcgen05 access of this CTA is done before the dealloc
  tc_fence_before();
  __syncthreads();
  if (warp == kPfMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tbase, kPfTmemCols);
  }
}

bool prefill_fast_supported(const AttnArgs& a) {
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0; };
  const int64_t pairs = (static_cast<int64_t>(a.max_query_len) + kPfPair - 1) / kPfPair;
  return (a.dtype == PKV_DTYPE_F16 || a.dtype == PKV_DTYPE_BF16) && a.head_dim == 64 &&
         a.block_size == 16 && a.max_query_len > 0 &&
         pairs * a.n_q_heads * a.n_seqs < (int64_t{1} << 31) &&
         (a.q_stride * 2) % 16 == 0 && (a.out_stride * 2) % 16 == 0 && al(a.q, 16) &&
         al(a.out, 16) && al(a.k_pool, 16) && al(a.v_pool, 16) &&
         a.scale > 0.f && static_cast<int64_t>(a.n_tokens) + kPfPair < (int64_t{1} << 31);
}

// fp8 pools on the tensor cores with the in-kernel conversion: fp16 queries,
// up to kPf8MaxKvHeads KV heads, scale rows bulk-copyable
bool prefill_fp8_tc_supported(const AttnArgs& a) {
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & (m - 1)) == 0; };
  return a.k_scale != nullptr && a.v_scale != nullptr && a.dtype == PKV_DTYPE_F16 &&
         a.n_kv_heads <= kPf8MaxKvHeads && al(a.k_scale, 16) && al(a.v_scale, 16) &&
         prefill_fast_supported(a);
}

namespace {
std::mutex g_pf_mu;
int g_pf_state[64][4] = {};  // [device][dtype x fp8]: 0 unchecked, 1 ready, -1 split does not fit
}  // namespace

cudaError_t launch_prefill_fast(const AttnArgs& a, const CUtensorMap* qmap, const CUtensorMap* kmap,
                                const CUtensorMap* vmap, cudaStream_t stream) {
  if (a.n_seqs == 0 || a.n_tokens == 0) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // fp8 pools (the scales given): the kernel converts the e4m3 tiles itself
  const bool fp8 = a.k_scale != nullptr;
  if (fp8 && !prefill_fp8_tc_supported(a)) return cudaErrorNotSupported;
  auto kern = fp8 ? paged_prefill_tc_kernel<__half, true>
              : a.dtype == PKV_DTYPE_F16 ? paged_prefill_tc_kernel<__half, false>
                                         : paged_prefill_tc_kernel<__nv_bfloat16, false>;
  const int smem = fp8 ? kPfSmemBytesFp8 : kPfSmemBytes;
  {
    std::lock_guard<std::mutex> lk(g_pf_mu);
    const int k = fp8 ? 2 : a.dtype == PKV_DTYPE_F16 ? 0 : 1;
    int state = dev < 64 ? g_pf_state[dev][k] : 0;
    if (state == 0) {
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return e;
      state = fa.numRegs * kPfThreads >= kPfRegSplit ? 1 : -1;
      if (state == 1) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
      }
      if (dev < 64) g_pf_state[dev][k] = state;
    }
    // a build whose launch register count cannot fund the split runs the
    // CUDA-core kernel instead
    if (state != 1) return launch_generic_attention(a, stream);
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
  p.n_seqs = a.n_seqs;
  p.n_q_heads = a.n_q_heads;
  p.n_pairs = (a.max_query_len + kPfPair - 1) / kPfPair;
  p.order_by_length = a.n_seqs <= kPfOrderMaxSeqs ? 1 : 0;
  p.group = a.n_q_heads / a.n_kv_heads;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  p.err = a.err;
  p.k_scale = a.k_scale;
  p.v_scale = a.v_scale;
  p.n_kv_heads = a.n_kv_heads;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.n_pairs * a.n_q_heads * a.n_seqs));
  cfg.blockDim = dim3(kPfThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, *qmap, *kmap, *vmap, p);
}

}  // namespace pkv
