// Thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers, TMA (cp.async.bulk.tensor), and the 5th-generation tensor core
// (tcgen05: TMEM allocation, MMA, commit, TMEM loads/stores).
//
// Every spin-wait here is bounded: after kWaitLimitCycles of polling it
// records an error code in the caller-supplied device word and returns false,
// so a kernel can unwind (free TMEM, drain its own copies) instead of hanging.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tfx {

// ~1.1 s at 1.9 GHz. A legitimate hand-off between warps of one CTA takes
// microseconds, so reaching this means a protocol bug, never slowness.
constexpr long long kWaitLimitCycles = 2000000000LL;

// Device error codes written to the error word (first writer wins).
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,      // consumer gave up waiting for a TMA stage
  kDevTimeoutEmpty = 2,     // producer gave up waiting for a free stage
  kDevTimeoutAccum = 3,     // epilogue gave up waiting for the accumulator
  kDevTimeoutAccumFree = 4, // MMA warp gave up waiting for a free accumulator
  kDevTimeoutOther = 5,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------- programmatic dependent launch
// Blocks until the previous grid in the stream has completed and its memory
// is visible (returns at once when there is none). Called by every thread of
// every kernel before its first global-memory access and before TMEM is
// allocated: a CTA that holds TMEM then never waits on an earlier grid, so
// an earlier grid's CTA sharing the SM always gets its TMEM and finishes.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next grid in the stream be scheduled (it still waits for this
// grid's completion in its own grid_dep_wait).
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
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

// Wait until the phase with the given parity has completed, polling for at
// most limit_cycles; on timeout record `code` in *err and return false.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, int code,
                                              long long limit_cycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > limit_cycles) {
      record_error(err, code);
      return false;
    }
  }
}

// Wait until the phase with the given parity has completed. Bounded.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  return mbar_wait_for(bar, parity, err, code, kWaitLimitCycles);
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps until it completes or kSuspendHintNs pass, instead of returning
// after the short default limit.
constexpr uint32_t kSuspendHintNs = 50000;
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// mbar_wait whose polls sleep (at most kSuspendHintNs each, same overall
// bound). For kernels whose waiting warps share SM sub-partitions with
// busy ones: a sleeping poller takes almost no issue slots from them.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* err,
                                                int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return true;
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(err, code);
      return false;
    }
  }
}

// -------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Untiled bulk copy global -> shared, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Make generic-proxy writes to shared memory visible to the async proxy
// (TMA store, tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Hint: bring [p, p + bytes) of global memory into L2 (no shared memory, no
// completion to wait for). p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(p)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one full warp. ncols is a power of two >= 32.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
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

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16/bf16 in, fp32 acc).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same, with the A operand read from TMEM (row i of A in TMEM lane i).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// TMEM lane (base_lane + t), columns [col, col+32).
// All tcgen05.ld / tcgen05.st here are .sync.aligned: every lane of the warp
// must execute them together, so callers keep them out of per-lane branches
// and predicate only the global-memory side.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld1(uint32_t taddr, uint32_t& r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(r) : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle that TMA's CU_TENSOR_MAP_SWIZZLE_128B writes: rows of
// 64 fp16 (128 B), 8-row atoms of 1024 B stacked contiguously.
//   bits  0-13 start address >> 4
//   bits 16-29 leading byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout (2 = 128-byte swizzle)
// Advancing along K inside the 128-byte row is done by adding the byte
// offset to the start address; the tile base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Shared-memory descriptor for an MN-major operand with the 128-byte swizzle:
// the tile is stored as rows along K (one 128-byte row = 64 fp16 along M/N),
// 8-row atoms of 1024 B stacked along K (stride byte offset 1024), and
// further 64-wide blocks along M/N `lbo_bytes` apart (leading byte offset).
// This is exactly a row-major [K rows x 64 cols] tile written by TMA with
// CU_TENSOR_MAP_SWIZZLE_128B, e.g. a V tile [keys x head_dim] used as the B
// operand of P.V. Advancing K by 16 adds 16 rows = 2048 bytes.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t smem_addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp16 A and B (both K-major), fp32 D,
// shape M x N (M in {64,128}, N a multiple of 16 up to 256).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (0u << 7) | (0u << 10)                   // A, B format: f16
         | (0u << 15) | (0u << 16)                  // A, B K-major
         | (static_cast<uint32_t>(n >> 3) << 17)    // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);   // M >> 4
}

// Same, with the B operand MN-major (bit 16).
__host__ __device__ constexpr uint32_t idesc_f16_f32_bmn(int m, int n) {
  return idesc_f16_f32(m, n) | (1u << 16);
}

// ------------------------------------------------------------ conversions
__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 2^x with the hardware approximation (ex2.approx.ftz.f32; flushes
// denormal results to zero, exact 0 for -inf).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------- packed fp32 pairs (sm_100)
// Two fp32 values in one 64-bit register pair; add/sub/fma.rn.f32x2 do both
// lanes in one instruction (half the issue slots of scalar FADD/FFMA).
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
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// Exact-erf GELU of a pair, x * Phi(x) = x/2 * (1 + erf(x / sqrt 2)), on the
// FMA pipe only (no MUFU). With z = x / sqrt 2: erf(z) = zc * Q(t), zc = z
// clamped to [-3.5, 3.5] (1 - erf(3.5) = 7.4e-7) and t = zc^2 * 2/3.5^2 - 1 in
// [-1, 1], where the monomial basis is well conditioned for fp32. Q (degree
// 9) is a fit computed for this file: Lawson's iteratively reweighted least
// squares towards the minimax absolute error of erf on [0, 3.5]. Evaluated
// as x * (1/2 + xc * Q'(t)) with xc = x clamped to +-3.5 sqrt 2, t = xc^2 /
// 3.5^2 - 1 and Q' = Q / (2 sqrt 2) (13 paired FMA-pipe operations). In fp32:
// |erf error| <= 2.6e-5, so |GELU error| <= 1.3e-5 * |x| (the fp16 the result
// is stored in rounds by 2.4e-4 relative: 6.5e-5 against 1.2e-3 at |x| = 5).
__device__ __forceinline__ uint64_t gelu_poly_f2(uint64_t x) {
  constexpr float kClamp = 4.949747562408447f;  // 3.5 * sqrt 2
  float x0, x1;
  f2_unpack(x, x0, x1);
  const uint64_t xc = f2_pack(fminf(fmaxf(x0, -kClamp), kClamp), fminf(fmaxf(x1, -kClamp), kClamp));
  const uint64_t t = f2_fma(xc, f2_mul(xc, f2_pack(0.08163265138864517f, 0.08163265138864517f)),
                            f2_pack(-1.0f, -1.0f));
  constexpr float kQ[10] = {0.14279407262802124f,  -0.07094885408878326f,
                            0.05169449374079704f,  -0.0406164787709713f,
                            0.03290337696671486f,  -0.022924380376935005f,
                            0.011054934933781624f, -0.009290049783885479f,
                            0.011502576991915703f, -0.005157033912837505f};
  uint64_t p = f2_pack(kQ[9], kQ[9]);
#pragma unroll
  for (int k = 8; k >= 0; --k) p = f2_fma(p, t, f2_pack(kQ[k], kQ[k]));
  return f2_mul(x, f2_fma(xc, p, f2_pack(0.5f, 0.5f)));
}

// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair, on the FMA pipe instead of the MUFU unit. Cody-Waite range
// reduction x = n + f with n = round(x) (the 1.5 * 2^23 rounding-constant
// trick, exact in round-to-nearest for |x| < 2^22) and |f| <= 1/2; 2^f from a
// degree-3 polynomial whose coefficients are a relative-error minimax fit on
// [-1/2, 1/2] computed for this file (Lawson's iteratively reweighted least
// squares; max relative error 7.5e-5, below half an fp16 ulp, 2.4e-4); 2^n is
// applied by adding n to the exponent field. Inputs are clamped to >= -126 so
// the exponent never underflows (results below 2^-126 only feed fp16 P
// values, where they round to 0); -inf gives 2^-126. Inputs must be <= 127.
__device__ __forceinline__ uint64_t exp2_poly_f2(uint64_t x) {
  float x0, x1;
  f2_unpack(x, x0, x1);
  const uint64_t xc = f2_pack(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
  const uint64_t kRound = f2_pack(12582912.0f, 12582912.0f);  // 1.5 * 2^23
  const uint64_t j = f2_add(xc, kRound);                        // n in the low mantissa bits
  const uint64_t f = f2_sub(xc, f2_sub(j, kRound));             // x - n
  uint64_t p = f2_fma(f, f2_pack(0.055171433836221695f, 0.055171433836221695f),
                      f2_pack(0.24261081218719482f, 0.24261081218719482f));
  p = f2_fma(p, f, f2_pack(0.6932609677314758f, 0.6932609677314758f));
  p = f2_fma(p, f, f2_pack(0.9999281167984009f, 0.9999281167984009f));
  float p0, p1, j0, j1;
  f2_unpack(p, p0, p1);
  f2_unpack(j, j0, j1);
  const uint32_t r0 = __float_as_uint(p0) + (__float_as_uint(j0) << 23);
  const uint32_t r1 = __float_as_uint(p1) + (__float_as_uint(j1) << 23);
  return f2_pack(__uint_as_float(r0), __uint_as_float(r1));
}

// ------------------------------------------------- thread-block clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the same shared-memory location in CTA `rank`
// of this cluster (distributed shared memory).
__device__ __forceinline__ uint32_t mapa_shared(uint32_t cta_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(cta_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t cluster_addr, uint32_t a, uint32_t b,
                                              uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(a),
               "r"(b), "r"(c), "r"(d)
               : "memory");
}

// Orders this thread's generic-proxy writes to shared::cluster memory (its
// own or a peer's) before later async-proxy (tensor core, TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_cluster() {
  asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
}

// Arrive on an mbarrier in another CTA of the cluster (release at cluster
// scope: this thread's earlier writes are visible to whoever acquires it).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   cluster_bar_addr)
               : "memory");
}

// Bounded wait (acquire at cluster scope) on a local mbarrier that a peer
// CTA arrives on; suspends between polls like mbar_wait_sleep.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err,
                                                  int code) {
  const long long t0 = clock64();
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kWaitLimitCycles) {
      record_error(err, code);
      return false;
    }
  }
}

// Cluster-wide barrier of every thread of every CTA in the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Per-warpgroup register limits (all 128 threads of a warpgroup execute
// them together). The block's pool is its launch allocation (threads x
// registers per thread); .inc blocks until other warpgroups' .dec have freed
// enough of it, so the split must add up to the launch allocation.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Named barrier over `count` threads (a multiple of 32) with id `id` (1..15).
// Arrive on named barrier `id` without waiting (pairs with named_bar_sync
// by the other threads of the `count`).
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}


}  // namespace tfx
