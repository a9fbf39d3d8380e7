// Device-side building blocks for the sm_100a kernels of heiretsu_b200.
//
// Everything here is a thin wrapper over one PTX instruction (or a short
// sequence) of the Blackwell execution model: mbarriers, TMA tensor copies
// (never with cluster multicast), tcgen05 tensor-memory allocation, MMA,
// commit and loads, and the UMMA shared-memory / instruction descriptors.
//
// Every wait in this file is bounded: it gives up after HB_WAIT_TIMEOUT_NS of
// %globaltimer time, records an error code in the device status word and
// returns false, so that a kernel whose partner never arrives returns instead
// of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#ifndef HB_WAIT_TIMEOUT_NS
#define HB_WAIT_TIMEOUT_NS 2000000000ull  // 2 s: legitimate waits are microseconds
#endif

namespace hb {

// ---------------------------------------------------------------------------
// Device status word (one per device, allocated by the host runtime).
// Codes: 0 ok; 1 mbarrier timeout; 2 peer-flag timeout; 3 bad argument.
// ---------------------------------------------------------------------------
enum StatusCode : int { kOk = 0, kMbarTimeout = 1, kPeerTimeout = 2, kBadArg = 3 };

__device__ __forceinline__ void record_error(int* status, int code, int where) {
  if (status != nullptr) {
    // Keep the first error; encode the site in the upper bits.
    atomicCAS(status, 0, code | (where << 8));
  }
}

// Debug-build invariant checks (compile with -DHB_DEBUG): evaluate to the
// condition; a violated check records kBadArg with its site in the status
// word, and the caller skips the access. Release builds compile them out.
#ifdef HB_DEBUG
#define HB_DCHECK(cond, status, site) \
  ((cond) ? true : (::hb::record_error((status), ::hb::kBadArg, (site)), false))
#else
#define HB_DCHECK(cond, status, site) true
#endif

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > HB_WAIT_TIMEOUT_NS) {
      record_error(status, kMbarTimeout, where);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tiled tensor copies, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Make generic-proxy writes to shared memory visible to the async proxy
// (TMA / tensor core) before they are consumed there.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk tensor stores / reductions from shared memory (epilogues). The source
// tile must be written with generic stores, then fence_proxy_async_smem()
// by the writing threads, before one thread issues the copy.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
// global += smem tile (fp32 add performed at L2).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1,
                                                  int c2) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk copy of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk copy of this thread has completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, loads
// ---------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to shared memory at `dst`. Must be executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
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

// D[tmem] (+)= A[smem] * B[smem]^T, bf16/f16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Load 32 consecutive fp32 columns of this warp's 32 TMEM lanes: thread t
// receives row (lane_base + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Split form of tmem_ld32 for overlapping several loads: issue without
// waiting, then wait once. The wait names the destination registers as
// in/out operands, so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}
// After one wait covering several issued loads, pin the other arrays' registers too.
__device__ __forceinline__ void tmem_pin_regs(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Store 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (sm_100 encoding)
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor for a 128-byte-swizzled tile.
//   bits [0,14)  start address >> 4
//   bits [16,30) leading-dimension byte offset >> 4
//   bits [32,46) stride-dimension byte offset >> 4
//   bits [46,48) descriptor version (1 on sm_100)
//   bits [61,64) layout: 2 = SWIZZLE_128B
// K-major tile (rows of 64 bf16 = 128 B, 8-row swizzle atoms of 1024 B):
//   LBO unused (encoded 1), SBO = 1024 B.
// MN-major tile (atoms of 64 MN-elements x 8 K-rows, 1024 B; atoms along K
// at 1024 B, atoms along MN at `mn_atom_stride` bytes):
//   LBO = mn_atom_stride, SBO = 1024 B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   [4,6) D format (1 = f32); [7,10) A format; [10,13) B format (0 f16, 1 bf16)
//   [15] A major (1 = MN-major); [16] B major; [17,23) N >> 3; [24,29) M >> 4
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, bool a_mn, bool b_mn, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((static_cast<uint32_t>(N) >> 3) << 17) |
         ((static_cast<uint32_t>(M) >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------
// GELU, tanh approximation (the GELU(approximate="tanh") of the model):
//   gelu(x) = 0.5 x (1 + tanh(u)),  u = sqrt(2/pi) (x + 0.044715 x^3).
// Evaluated through the identity 1 + tanh(u) = 2 sigmoid(2u), so
//   gelu(x) = x * s,  s = 1 / (1 + 2^(-2u log2 e)).
// The exponential is one ex2.approx; the reciprocal stays off the
// transcendental unit (which the epilogue's bf16 conversions also use): an
// initial estimate by integer subtraction on the float's bit pattern,
// refined by two Newton steps r <- r (2 - d r).
//
// The seed constant, derived here: write d = 2^E (1 + m), m in [0, 1), and
// K = 0x7E800000 + c * 2^23 (0x7E800000 is exponent field 253). Then
// K - bits(d) decodes to 2^(-E-1) (1 + c - m) when m <= c, and, after the
// borrow from the exponent field, to 2^(-E-2) (2 + c - m) when m > c. So
//   r d = (1 + c - m)(1 + m) / 2   or   (2 + c - m)(1 + m) / 4.
// The largest |r d - 1| is (1 - c)/2 (at m = 0 and m -> 1) or
// (1 + c/2)^2 / 2 - 1 (the peak at m = c/2). Equal ripple gives
// c^2 + 8c - 8 = 0, c = 2 sqrt(6) - 4, K = 0x7E800000 + round(c * 2^23)
// = 0x7EF311C3, and a seed error of at most (5 - 2 sqrt(6)) / 2 < 5.06%
// (the same in every binade). Each Newton step squares the relative error:
// < 2.6e-3, then < 7e-6 -- far below bf16 resolution. The exponent is
// clamped at 64 so d stays finite; gelu -> x * 2^-64 ~ 0 there.
__device__ __forceinline__ float sigmoid_2u(float u) {
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(fminf(-2.8853900817779268f * u, 64.f)));  // -2 log2(e) u
  const float d = 1.f + e;
  float r = __int_as_float(0x7EF311C3 - __float_as_int(d));
  r = r * fmaf(-d, r, 2.f);
  r = r * fmaf(-d, r, 2.f);
  return r;
}

// 2^x on the FMA / integer pipes, for x in [-125, 64] (clamped), to take part
// of the exponentials off the transcendental unit (whose throughput the
// epilogue's 16-bit conversions also use). Derived here:
//   n = nearest integer to x: adding 1.5 * 2^23 (0x4B400000) leaves n in the
//   low mantissa bits of t = x + 1.5 * 2^23, and t - 1.5 * 2^23 is n as a float;
//   f = x - n lies in [-1/2, 1/2];
//   2^f = e^(f ln 2) by its Taylor series to degree 5, coefficients (ln 2)^k / k!;
//   the Lagrange remainder bounds the relative error: with |f ln 2| <= ln(2)/2,
//   |R| / 2^f <= (ln(2)/2)^6 / 6! * e^(ln 2) < 5e-6;
//   2^x = 2^f * 2^n: n is added to the exponent field of 2^f (which lies in
//   [0.70, 1.42], so the result's exponent stays normal for n >= -125).
__device__ __forceinline__ float exp2_fma(float x) {
  x = fminf(fmaxf(x, -125.f), 64.f);
  const float t = x + 12582912.f;
  const float f = x - (t - 12582912.f);
  float p = fmaf(f, 1.3333558146428443e-3f, 9.6181291076284772e-3f);  // (ln 2)^5/5!, (ln 2)^4/4!
  p = fmaf(f, p, 5.5504108664821580e-2f);                             // (ln 2)^3/3!
  p = fmaf(f, p, 2.4022650695910071e-1f);                             // (ln 2)^2/2!
  p = fmaf(f, p, 6.9314718055994531e-1f);                             // ln 2
  p = fmaf(f, p, 1.f);
  return __int_as_float(__float_as_int(p) + ((__float_as_int(t) - 0x4B400000) << 23));
}

// sigmoid(2u) as sigmoid_2u, with the exponential from exp2_fma.
__device__ __forceinline__ float sigmoid_2u_fma(float u) {
  const float d = 1.f + exp2_fma(-2.8853900817779268f * u);
  float r = __int_as_float(0x7EF311C3 - __float_as_int(d));
  r = r * fmaf(-d, r, 2.f);
  r = r * fmaf(-d, r, 2.f);
  return r;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return x * sigmoid_2u(k0 * fmaf(k1 * x, x * x, x));
}
// The same function with its exponential on the FMA pipe (epilogues alternate the two).
__device__ __forceinline__ float gelu_tanh_fma(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  return x * sigmoid_2u_fma(k0 * fmaf(k1 * x, x * x, x));
}

// The same function through the hardware tanh approximation (tanh.approx.f32,
// relative error about 2^-11, below the 16-bit outputs' rounding):
//   gelu(x) = h + h t,  h = x / 2,  t = tanh(x (k0 + k0 k1 x^2)).
__device__ __forceinline__ float tanh_approx(float u) {
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return t;
}
__device__ __forceinline__ float gelu_tanh_mufu(float x) {
  const float k0 = 0.7978845608028654f;
  const float k01 = 0.7978845608028654f * 0.044715f;
  const float h = 0.5f * x;
  const float t = tanh_approx(x * fmaf(k01, x * x, k0));
  return fmaf(h, t, h);
}

// d/dx gelu(x) = s + 2 x s (1 - s) du/dx,  du/dx = sqrt(2/pi) (1 + 3 * 0.044715 x^2)
// (product rule on x * sigmoid(2u); equals 0.5(1+t) + 0.5 x (1-t^2) du/dx with t = tanh u).
__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  const float x2 = x * x;
  const float s = sigmoid_2u(k0 * fmaf(k1 * x, x2, x));
  const float du = k0 * fmaf(3.f * k1, x2, 1.f);
  return fmaf(2.f * x * s * (1.f - s), du, s);
}
__device__ __forceinline__ float gelu_tanh_grad_fma(float x) {
  const float k0 = 0.7978845608028654f;
  const float k1 = 0.044715f;
  const float x2 = x * x;
  const float s = sigmoid_2u_fma(k0 * fmaf(k1 * x, x2, x));
  const float du = k0 * fmaf(3.f * k1, x2, 1.f);
  return fmaf(2.f * x * s * (1.f - s), du, s);
}
// 0.5 (1 + t) + 0.5 x (1 - t^2) du/dx with t from tanh.approx.
__device__ __forceinline__ float gelu_tanh_grad_mufu(float x) {
  const float k0 = 0.7978845608028654f;
  const float k01 = 0.7978845608028654f * 0.044715f;
  const float x2 = x * x;
  const float t = tanh_approx(x * fmaf(k01, x2, k0));
  const float du = fmaf(3.f * k01, x2, k0);
  return fmaf(0.5f * x * fmaf(-t, t, 1.f), du, fmaf(0.5f, t, 0.5f));
}

// Packed fp32 pairs: sm_100 executes add / mul / fma on two fp32 values in
// one instruction (PTX .f32x2); the pair lives in a 64-bit register.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 16-bit storage formats. Activations and weight shadows are bf16 under
// --amp bf16 and fp16 under --amp fp16; kernels take the format as a template
// argument (F16) or, where one compiled kernel serves both, as a flag.
template <bool F16>
__device__ __forceinline__ uint32_t pack16(float a, float b) {
  return F16 ? pack_f16(a, b) : pack_bf16(a, b);
}
__device__ __forceinline__ uint32_t pack16(float a, float b, bool f16) {
  return f16 ? pack_f16(a, b) : pack_bf16(a, b);
}
// Low / high element of a packed pair as fp32.
template <bool F16>
__device__ __forceinline__ float lo16(uint32_t w) {
  if constexpr (F16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
  } else {
    return __uint_as_float(w << 16);
  }
}
template <bool F16>
__device__ __forceinline__ float hi16(uint32_t w) {
  if constexpr (F16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
  } else {
    return __uint_as_float(w & 0xFFFF0000u);
  }
}
template <bool F16>
__device__ __forceinline__ float to_f32(uint16_t v) {
  if constexpr (F16) {
    return __half2float(__ushort_as_half(v));
  } else {
    return __uint_as_float(static_cast<uint32_t>(v) << 16);
  }
}
template <bool F16>
__device__ __forceinline__ uint16_t from_f32(float x) {
  if constexpr (F16) {
    return __half_as_ushort(__float2half_rn(x));
  } else {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
}

// x rounded to the 16-bit format (nearest even) and widened back to fp32.
template <bool F16>
__device__ __forceinline__ float round16(float x) {
  return to_f32<F16>(from_f32<F16>(x));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace hb
