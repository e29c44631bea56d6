// Inline-PTX building blocks for the sm_100a kernels: mbarriers (with bounded waits), TMA tile
// loads, and the tcgen05 tensor-memory / tensor-core instructions.
//
// Every wait in this library is bounded: after LBQ_SPIN_LIMIT polls it records an error code in
// the kernel's status word, raises the CTA's abort flag and returns false, so that a broken
// pipeline ends the kernel with an error the host can read instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#ifndef LBQ_SPIN_LIMIT
#define LBQ_SPIN_LIMIT (1u << 26)
#endif
#ifndef LBQ_WAIT_LIMIT_NS
#define LBQ_WAIT_LIMIT_NS 4000000000ull   // 4 s of wall time per wait, measured on %globaltimer
#endif

namespace lbq {

// Status codes written to the device status word (also returned by lbq_device_status()).
enum DeviceStatus : int {
  kDevOk = 0,
  kDevTimeoutQ = 0x101,      // Q tile never arrived
  kDevTimeoutKV = 0x102,     // producer: K/V stage never released / consumer: never filled
  kDevTimeoutS = 0x103,      // softmax: S tile never completed
  kDevTimeoutP = 0x104,      // MMA: P tile never written
  kDevTimeoutO = 0x105,      // O accumulator never completed
  kDevTimeoutPeerStats = 0x201,  // sequence split: a rank's share statistics never arrived
  kDevTimeoutPeerData = 0x202,   // sequence split: a rank's K/V share never arrived
  kDevBadStatsRow = 0x301,       // debug build: block-statistics row outside the table
  kDevBadSourceToken = 0x302,    // debug build: quantizer source token below 0
  kDevBadTile = 0x303,           // debug build: key tile outside its code segment
  kDevBadOwner = 0x304,          // debug build: key-range partial outside the owner's receive slot
};

// Debug builds (-DLBQ_DEBUG=1, liblbq_debug.so) check the index arithmetic at the places the kDevBad*
// codes name: a failed check records its code in the status word (the first failure wins) and the
// caller clamps or skips the access; nothing traps. Release builds compile every check to `true`
// without evaluating its condition.
#if defined(LBQ_DEBUG) && LBQ_DEBUG
__device__ __forceinline__ bool lbq_check(bool ok, int* status, int code) {
  if (!ok && status != nullptr) atomicCAS(status, 0, code);
  return ok;
}
#define LBQ_CHECK(cond, status, code) ::lbq::lbq_check((cond), (status), (code))
#else
#define LBQ_CHECK(cond, status, code) true
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// True in exactly one lane of the (converged) warp. A role that issues TMA copies or tcgen05 MMAs runs
// as a whole warp and issues under elect_one(): its descriptors and addresses are then computed
// uniformly by the warp and stay in uniform registers.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "@px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
#ifndef LBQ_TRY_WAIT_HINT_NS
#define LBQ_TRY_WAIT_HINT_NS 0
#endif
// Waits until the phase with `parity` completes or the instruction's own time limit runs out (with
// LBQ_TRY_WAIT_HINT_NS > 0: a suspend-time hint of that many ns); returns whether the phase completed.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
#if LBQ_TRY_WAIT_HINT_NS > 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(uint32_t(LBQ_TRY_WAIT_HINT_NS))
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait. Returns false (and records `code`) when the CTA was aborted, or when the phase has
// not completed after LBQ_WAIT_LIMIT_NS of wall time or LBQ_SPIN_LIMIT polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1; i < LBQ_SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((i & 255) == 0 && globaltimer_ns() - t0 > LBQ_WAIT_LIMIT_NS) break;
  }
  *abort_flag = 1;
  if (status) atomicCAS(status, 0, code);
  return false;
}
#ifndef LBQ_ROLE_SLEEP_NS
#define LBQ_ROLE_SLEEP_NS 64
#endif
// mbar_wait for the TMA producer warps and the issuers' waits that are not on the softmax's path, which
// share their SM sub-partition with softmax warps: between polls the warp sleeps LBQ_ROLE_SLEEP_NS, so
// that its polling does not take their issue slots.
__device__ __forceinline__ bool mbar_wait_role(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status,
                                               int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1; i < LBQ_SPIN_LIMIT; ++i) {
#if LBQ_ROLE_SLEEP_NS > 0
    __nanosleep(LBQ_ROLE_SLEEP_NS);
#endif
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if ((i & 255) == 0 && globaltimer_ns() - t0 > LBQ_WAIT_LIMIT_NS) break;
  }
  *abort_flag = 1;
  if (status) atomicCAS(status, 0, code);
  return false;
}
// Bounded wait used while draining after an abort (ignores the abort flag).
__device__ __forceinline__ void mbar_drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < LBQ_SPIN_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 255) == 0 && globaltimer_ns() - t0 > LBQ_WAIT_LIMIT_NS) return;
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 3-D tiled load (no multicast) into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05 (tensor memory)
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once all tcgen05 async operations issued so far by this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> fp32.
__device__ __forceinline__ void mma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Makes this thread's generic-proxy shared-memory writes visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of 128 bytes, 8-row
// core groups 1024 bytes apart (the layout a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes).
// Bits: [0,14) start>>4, [16,30) LBO>>4 (unused for swizzled K-major, 1), [32,46) SBO>>4,
// [46,48) version 1 (sm_100), [61,64) layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptors (M=128, both operands K-major, dense).
//   [4,6) D format (1 = f32, 2 = s32), [7,10) A format, [10,13) B format,
//   [17,23) N>>3, [24,29) M>>4.
constexpr uint32_t idesc_m128(uint32_t n, uint32_t dfmt, uint32_t afmt, uint32_t bfmt) {
  return (dfmt << 4) | (afmt << 7) | (bfmt << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}
constexpr uint32_t kIdescQK = idesc_m128(128, 2, 1, 1);   // s32 <- s8 x s8, N = 128 keys
constexpr uint32_t kIdescPV = idesc_m128(128, 1, 0, 0);   // f32 <- e4m3 x e4m3, N = 128 channels

// Warp-collective TMEM load: thread i of the warp reads lane (lane_base + i), 32 consecutive
// 32-bit columns starting at the column in `taddr`.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Waits for this thread's TMEM loads and ties the 32 destination registers to the wait, so that the
// compiler cannot move a use of them above it.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}
// No instruction: orders the 32 registers after the preceding volatile asm (a second tmem_ld_wait).
__device__ __forceinline__ void reg_anchor(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t (&r)[8]) { tmem_st8(taddr, r); }
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]);
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t (&r)[16]) { tmem_st16(taddr, r); }
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- register reallocation
// Every warp of a warpgroup executes the same setmaxnreg. The per-thread counts of all warpgroups of a
// CTA must add up to at most what the CTA was launched with (threads x registers at launch), or an
// increase waits forever.
template <uint32_t N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- numerics
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Two fp32 -> two e4m3 (RN, saturate to +-448) packed in 16 bits, `lo` in the low byte.
__device__ __forceinline__ uint32_t pack_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// Two floats to an activation pair (dtype 0: bf16, 1: fp16; round to nearest even), `lo` in the low
// 16 bits.
__device__ __forceinline__ uint32_t pack_act2(float lo, float hi, int dtype) {
  if (dtype) {
    const __half2 p = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
  }
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}
// One 256-bit global store of eight 32-bit words (the address 32-byte aligned).
__device__ __forceinline__ void st_global_v8(void* p, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}
// The two activations of a 32-bit pair (dtype 0: bf16, 1: fp16) as floats (exact).
__device__ __forceinline__ void act2_to_f32(uint32_t w, int dtype, float& lo, float& hi) {
  if (dtype) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
    lo = f.x;
    hi = f.y;
  } else {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  }
}
// ---- packed fp32 pairs (sm_100 f32x2 instructions: one issue slot for two lanes of work)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair on the FMA pipe (no MUFU): x is clamped to >= -125, split as x = j + f with
// j = round(x) (magic-number rounding) and f in [-0.5, 0.5]; 2^f is a degree-3 polynomial fitted
// here to minimise the maximum relative error on [-0.5, 0.5] (7.5e-5, iteratively reweighted
// least squares), and j is added to the exponent field with an integer multiply-add.
__device__ __forceinline__ uint64_t exp2_poly_x2(float x0, float x1) {
  constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
  x0 = fmaxf(x0, -125.f);
  x1 = fmaxf(x1, -125.f);
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t t = f2_add(x, f2_pack(kMagic, kMagic));
  const uint64_t j = f2_add(t, f2_pack(-kMagic, -kMagic));
  const uint64_t f = f2_fma(j, f2_pack(-1.f, -1.f), x);
  uint64_t p = f2_fma(f2_pack(5.517166853e-02f, 5.517166853e-02f), f, f2_pack(2.426111400e-01f, 2.426111400e-01f));
  p = f2_fma(p, f, f2_pack(6.932609677e-01f, 6.932609677e-01f));
  p = f2_fma(p, f, f2_pack(9.999280572e-01f, 9.999280572e-01f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  // bits(t) << 23 == round(x) << 23 (mod 2^32): the magic's own bits shift out of the word.
  const uint32_t r0 = __float_as_uint(t0) * 8388608u + __float_as_uint(p0);
  const uint32_t r1 = __float_as_uint(t1) * 8388608u + __float_as_uint(p1);
  return f2_pack(__uint_as_float(r0), __uint_as_float(r1));
}


}  // namespace lbq
