// pkv_common.cuh -- shared device helpers for the paged-KV kernels (sm_100a).
//
// Element traits for fp32 / fp16 / bf16, the device error-flag helper, and
// thin inline-PTX wrappers for the Blackwell primitives the kernels use:
// mbarrier transaction barriers, TMA tensor loads (cp.async.bulk.tensor),
// ldmatrix and the m16n8k16 tensor-core MMA.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/pagedkv.h"

namespace pkv {

// ----------------------------------------------------------------------------
// element traits
// ----------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// pack two floats into one 32-bit register of 16-bit elements (lo = first)
template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void raise_flag(int* err, int bits) {
  if (err != nullptr) atomicOr(err, bits);
}

// ----------------------------------------------------------------------------
// shared-memory addresses and mbarriers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
// make mbarrier initialisation visible to the async (TMA) proxy
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// e4m3 -> f16 on the integer pipes: the e4m3 fields moved into f16 position,
// which is the value times 2^-8 (exact, e4m3 subnormals included: they land
// on f16 subnormals).  The NaN encodings 0x7f / 0xff map to +-480; the
// quantising append never stores them.  Keeps conversions off the
// transcendental pipe, which the softmax's exponentials use.
// bytes 1 and 3 of x -> f16x2 (byte 1 in the low half)
__device__ __forceinline__ uint32_t e4m3_odd_h2(uint32_t x) {
  return (x & 0x80008000u) | ((x >> 1) & 0x3f803f80u);
}
// bytes 0 and 2 of x -> f16x2 (byte 0 in the low half)
__device__ __forceinline__ uint32_t e4m3_even_h2(uint32_t x) {
  const uint32_t z = (x << 7) & 0x7f807f80u;  // sign lands on bit 14 / 30
  return z + (z & 0x40004000u);               // ... and is carried to bit 15 / 31
}
// Bounded wait: gives up after ~2^31 SM cycles (about a second) and returns
// false, so a lost transaction can never hang the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) return false;
  }
  return true;
}
// Bounded wait for a device word that another agent (a copy engine) sets
// nonzero: acquire loads at GPU scope, a short sleep between them; gives up
// after ~2^31 SM cycles (about a second) and returns false.
__device__ __forceinline__ bool wait_word_nonzero(const int* w) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(w) : "memory");
  if (v != 0) return true;
  const long long t0 = clock64();
  do {
    if (clock64() - t0 > (1ll << 31)) return false;
    __nanosleep(256);
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(w) : "memory");
  } while (v == 0);
  return true;
}

// ----------------------------------------------------------------------------
// TMA: 3-D tiled tensor load global -> shared, completion on an mbarrier
// ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// L2 policy for data read exactly once (streamed KV): evict it first, so the
// small metadata every launch re-reads (block tables, lengths) stays cached
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// tma_load_3d with an L2 cache-policy hint
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int c0, int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}
// 1-D bulk copy global -> shared (16-byte aligned addresses, size multiple of 16)
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// warm L2 with `bytes` (multiple of 16) starting at a 16-byte aligned global address
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// order this thread's generic-proxy global writes before later async-proxy reads
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// order this thread's generic-proxy accesses before later async-proxy (TMA) accesses
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async;" ::: "memory");
}
// programmatic dependent launch: wait for the preceding grid / let dependents start
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------
// ldmatrix / mma.sync (m16n8k16, fp32 accumulate)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4],
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4],
                                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x with the SFU instruction (flush-to-zero; ex2(-inf) = +0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// transpose an 8x8 matrix of 16-bit elements held one row-pair per lane
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}


// ----------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core, tensor memory) -- cta_group::1 forms
// ----------------------------------------------------------------------------
// Allocate `ncols` (power of two >= 32) TMEM columns; the whole warp executes
// it and the TMEM base address is written to shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// order this thread's generic-proxy shared-memory writes before async-proxy reads
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor (sm_100 format): start address, leading and
// stride byte offsets (16-byte units), fixed version bits 46-48 = 0b001,
// base offset 0 (atoms 1024-byte aligned), swizzle mode in bits 61-63
// (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation: A/B format
// (0 = fp16, 1 = bf16), A/B major (0 = K-major, 1 = MN-major), N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t mma_idesc_f16(uint32_t ab_fmt, uint32_t a_mn_major,
                                                     uint32_t b_mn_major, uint32_t n, uint32_t m) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) |
         ((n >> 3) << 17) | ((m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]; issued by one thread.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (warp w: lanes 32w..32w+31).
// The registers are valid only after a tcgen05.wait::ld (tmem_wait_ld_regs below).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// tcgen05.wait::ld that also names the loaded registers as operands, so that no
// use of them can be scheduled above the wait; reg_after_wait() does the same
// for further register arrays loaded before that one wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
__device__ __forceinline__ void reg_after_wait(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// D[tmem] (+)= A[tmem] * B[smem]; A (M x 16 per instruction, K-major) is read
// from tensor memory: lane m = row m, 32-bit column c = elements 2c (low half)
// and 2c+1 (high half).  Issued by one thread.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Per-thread register budget of the executing warpgroup (all four warps of
// the warpgroup execute the same instruction).  .inc waits until the
// registers released by .dec of other warpgroups are available.
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// One leader lane of a converged warp (elect.sync over all 32 lanes; the same
// lane every time).  Issuing tcgen05.mma / TMA under this predicate from
// warp-converged code keeps their operands on the uniform datapath; under a
// per-lane test (lane == 0) every operand is moved there instruction by
// instruction, which costs several times the tensor core's own time for
// N <= 128 instructions.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// 2^x on the FMA pipe, for x <= ~16 (used beside ex2.approx to share the
// exponentials of a softmax between the MUFU and FMA pipes).
// Cody-Waite range reduction: t = x + 1.5 * 2^23 rounds x to the nearest
// integer n, held in t's low mantissa bits; f = x - n lies in [-1/2, 1/2].
// 2^f is a degree-3 polynomial fitted by Remez exchange to minimise the
// relative error on [-1/2, 1/2] (7.5e-5, against 4.9e-4 for rounding to
// fp16); 2^n is applied by adding n to the exponent field.  x is clamped at
// -125 so that the exponent field stays positive (p(f) can be below 1).
constexpr float kExp2C0 = 0x1.fff692p-1f;
constexpr float kExp2C1 = 0x1.62f31ap-1f;
constexpr float kExp2C2 = 0x1.f0de1ap-3f;
constexpr float kExp2C3 = 0x1.c3f760p-5f;
__device__ __forceinline__ float exp2_poly3(float x) {
  x = fmaxf(x, -125.f);
  const float t = __fadd_rn(x, 12582912.f);
  const float f = __fsub_rn(x, __fsub_rn(t, 12582912.f));
  const float p = fmaf(fmaf(fmaf(kExp2C3, f, kExp2C2), f, kExp2C1), f, kExp2C0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}
// exp2_poly3 of two values with the paired fp32 instructions of sm_100
// (__fadd2_rn / __ffma2_rn round each lane as __fadd_rn / fmaf do, so each
// lane's result equals exp2_poly3 bit for bit) at half the issue slots
__device__ __forceinline__ float2 exp2_poly3x2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 big = make_float2(12582912.f, 12582912.f), nbig = make_float2(-12582912.f, -12582912.f);
  const float2 t = __fadd2_rn(x, big);
  const float2 n = __fadd2_rn(t, nbig);
  const float2 f = __fadd2_rn(x, make_float2(-n.x, -n.y));
  float2 p = __ffma2_rn(make_float2(kExp2C3, kExp2C3), f, make_float2(kExp2C2, kExp2C2));
  p = __ffma2_rn(p, f, make_float2(kExp2C1, kExp2C1));
  p = __ffma2_rn(p, f, make_float2(kExp2C0, kExp2C0));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// ---- fp8 e4m3 KV: one scale per (token, KV head) row, absmax / 448
constexpr float kFp8Max = 448.f;  // largest finite e4m3 value
__device__ __forceinline__ float fp8_row_scale(float absmax) {
  return absmax > 0.f ? __fdiv_rn(absmax, kFp8Max) : 1.f;
}
// round to nearest even, saturating at +-448 (CUDA's conversion)
__device__ __forceinline__ uint8_t fp8_quantize(float x, float scale) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(__fdiv_rn(x, scale), __NV_SATFINITE, __NV_E4M3));
}
// Warp-collective fp8 append of one token: its n_heads rows of d values of
// type E (src, row h at src + h * d) quantised per row (scale = absmax / 448,
// e4m3 bytes, RNE, saturated) into dst (bytes, row h at dst + h * d) with the
// scales in sc[h].  Every lane of the warp must call it.
// two values as e4m3 bytes (lo in bits 0-7), rounded to nearest even and
// saturated at +-448: the rounding and saturation fp8_quantize asks of CUDA's
// conversion, two values per PTX cvt
__device__ __forceinline__ uint32_t e4m3x2_rn_sat(float lo, float hi) {
  unsigned short r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// four consecutive values of type E as floats (p aligned to 4 * sizeof(E))
template <typename E>
__device__ __forceinline__ void load4_f(const E* __restrict__ p, float* v) {
  if constexpr (sizeof(E) == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
  } else {
    const uint2 t = *reinterpret_cast<const uint2*>(p);
    const uint32_t w[2] = {t.x, t.y};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned short b = static_cast<unsigned short>(w[i >> 1] >> (16 * (i & 1)));
      if constexpr (std::is_same<E, __half>::value) v[i] = __half2float(__ushort_as_half(b));
      else v[i] = __bfloat162float(__ushort_as_bfloat16(b));
    }
  }
}
template <typename E>
__device__ __forceinline__ void fp8_store_token(const E* __restrict__ src, uint8_t* __restrict__ dst,
                                                float* __restrict__ sc, int n_heads, int d, int lane) {
  // Rows of 64 values (the pools' head_dim), aligned: two rows per pass, a
  // half-warp per row and four values per lane (one 8- or 16-byte load, one
  // 4-byte store, a 16-lane max).  Same per-value arithmetic as the general
  // loop below, so the same bytes and scales.
  if (d == 64 && (reinterpret_cast<uintptr_t>(src) & (4 * sizeof(E) - 1)) == 0 &&
      (reinterpret_cast<uintptr_t>(dst) & 3) == 0) {
    const int half = lane >> 4, l16 = lane & 15;
    for (int h0 = 0; h0 < n_heads; h0 += 2) {
      const int h = h0 + half;
      const bool on = h < n_heads;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (on) load4_f<E>(src + h * 64 + l16 * 4, v);
      float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (on) {
        const float s = fp8_row_scale(amax);
        const uint32_t q = e4m3x2_rn_sat(__fdiv_rn(v[0], s), __fdiv_rn(v[1], s)) |
                           (e4m3x2_rn_sat(__fdiv_rn(v[2], s), __fdiv_rn(v[3], s)) << 16);
        *reinterpret_cast<uint32_t*>(dst + h * 64 + l16 * 4) = q;
        if (l16 == 0) sc[h] = s;
      }
    }
    return;
  }
  for (int h = 0; h < n_heads; ++h) {
    float amax = 0.f;
    for (int i = lane; i < d; i += 32) amax = fmaxf(amax, fabsf(Elem<E>::to_f(src[h * d + i])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = fp8_row_scale(amax);
    for (int i = lane; i < d; i += 32) dst[h * d + i] = fp8_quantize(Elem<E>::to_f(src[h * d + i]), s);
    if (lane == 0) sc[h] = s;
  }
}

// exact: every e4m3 value is representable in fp16
__device__ __forceinline__ float fp8_to_float(uint8_t b) {
  return __half2float(__half(__nv_cvt_fp8_to_halfraw(b, __NV_E4M3)));
}

// three-input maximum (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

}  // namespace pkv
