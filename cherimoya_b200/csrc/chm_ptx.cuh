// chm_ptx.cuh -- inline-PTX helpers for sm_100a: tcgen05 MMA / TMEM,
// mbarriers with bounded waits, shared-memory operand descriptors.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

namespace chm {

// Iteration limit of every device-side wait. mbarrier.try_wait suspends the
// thread for a hardware-defined interval per call, so this bounds a wait to
// well under a minute even on a slow clock.
constexpr long long kWaitLimit = 200000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- launches
// Kernels launched with programmatic stream serialization may start while the
// previous kernel of the stream finishes; this waits until it has completed
// and its memory is visible. Everything before it may only touch this
// kernel's own shared memory / TMEM and data no earlier kernel of the same
// call writes.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async proxy (tcgen05.commit).
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(addr), "r"(parity)
      : "memory");
  return done != 0;
}

// Returns true when the phase with the given parity has completed, false if
// the bounded wait gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  for (long long it = 0; it < kWaitLimit; ++it) {
    if (mbar_try(addr, parity)) return true;
  }
  return false;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Wait bounded by wall time (kWaitNs) and by a block-wide abort flag that a
// thread whose own wait gave up sets: a stuck pipeline drains in about
// kWaitNs instead of each dependent wait running out in turn.
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity,
                                                    volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try(addr, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(addr, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kWaitNs) {
        *abort_flag = 1;
        return false;
      }
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// One arrive for the whole (converged) warp, from lane 0 after a warp
// barrier: the mbarrier's count is in warps.
__device__ __forceinline__ void mbar_arrive_warp(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// 2-D tiled TMA load (no multicast) into this CTA's shared memory; completes
// `bytes` of transaction count on `bar`. x must be 16-byte aligned in bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load (no multicast); coordinates (x, y, z) innermost first.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 16-byte asynchronous copy global -> shared (L2 only); with `valid` false
// the destination is zero-filled and nothing is read.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// wait until at most N committed groups of this thread are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 2-D tiled TMA store from this CTA's shared memory (bulk async group).
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(src)), "r"(x), "r"(y)
      : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory (no tensor map): `bytes` a
// multiple of 16, both addresses 16-byte aligned; completes `bytes` of
// transaction on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA store (bulk async group); elements outside the tensor are
// not written.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int x, int y,
                                             int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// wait until at most 0 bulk groups are still reading shared memory
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// wait until all bulk groups have completed (writes visible)
__device__ __forceinline__ void bulk_wait0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// named barrier over `count` threads (barrier 0 is __syncthreads)
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_async_smem() {
  // make generic-proxy shared-memory writes visible to the async proxy
  // (tcgen05.mma operand reads)
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- TMEM
// Allocation is warp-wide (.sync.aligned); the base address is written to
// shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// columns [col, col+32) of TMEM lane (lane_base + i). The load and its
// tcgen05.wait::ld are one asm statement, so no use of the destination
// registers can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns store (thread i -> lane base+i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns load, completed before returning.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns store.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// (tmem_ld32 already waits; kept as a no-op marker at the old call sites)
__device__ __forceinline__ void tmem_ld_wait() {}

// ---------------------------------------------------------------- MMA
// Shared-memory matrix descriptor, K-major operand in the canonical
// 128-byte-swizzled layout: rows of 128 bytes (64 bf16), 8-row groups of
// 1024 bytes (stride-dimension byte offset), swizzle mode 2, descriptor
// version 1 (sm_100).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);          // start address
  d |= static_cast<uint64_t>(1u) << 16;                        // LBO (unused, swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                // SBO = 1024 B
  d |= static_cast<uint64_t>(1u) << 46;                        // version
  d |= static_cast<uint64_t>(2u) << 61;                        // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 accumulate,
// both operands K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4)                                   // D format: f32
         | (1u << 7)                                 // A format: bf16
         | (1u << 10)                                // B format: bf16
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// D(tmem) (+)= A(smem) * B(smem)^T, issued by a single thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem)^T: A is read from tensor memory (16-bit
// elements packed two per 32-bit column, lane = row), issued by one thread.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when all previously issued MMAs of this thread are
// complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- layout
// Byte offset of element (row, k) in a K-major 128B-swizzled bf16 tile of
// `rows` rows: 64-wide K slabs, each `rows` x 128 B; the 16-byte chunk index
// inside a row is XORed with (row % 8).
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t k,
                                                          uint32_t rows) {
  const uint32_t slab = k >> 6;
  const uint32_t kk = k & 63u;
  const uint32_t chunk = (kk >> 3) ^ (row & 7u);
  return slab * rows * 128u + row * 128u + chunk * 16u + (kk & 7u) * 2u;
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU, tanh approximation: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
// kFast: hardware tanh.approx.f32 (bf16 mode). Otherwise the identity
// 0.5 (1 + tanh(u)) = 1 / (1 + exp(-2u)) with the CUDA exp/divide
// intrinsics (fp32 mode).
template <bool kFast>
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;            // sqrt(2/pi)
  const float k1 = 0.7978845608028654f * 0.044715f;
  const float u = x * fmaf(k1, x * x, k0);
  if (kFast) {
    const float hx = 0.5f * x;
    return fmaf(hx, tanh_fast(u), hx);
  } else {
    return __fdividef(x, 1.0f + __expf(-2.0f * u));
  }
}

// GELU(tanh) of two values in packed bf16x2 arithmetic (bf16 mode): the
// result is rounded to bf16 anyway, so u, tanh(u) and the final
// 0.5 x (1 + tanh u) are evaluated with bf16x2 FMAs and tanh.approx.bf16x2,
// three issue slots per value.
__device__ __forceinline__ uint32_t gelu_bf16x2(float z0, float z1) {
  uint32_t x, sq, t, u, th, hx, g;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(x) : "f"(z0), "f"(z1));
  const uint32_t k1 = 0x3D123D12u;   // bf16x2(0.0356774) = sqrt(2/pi) * 0.044715
  const uint32_t k0 = 0x3F4C3F4Cu;   // bf16x2(0.7978846) = sqrt(2/pi)
  const uint32_t half = 0x3F003F00u; // bf16x2(0.5)
  asm("mul.rn.bf16x2 %0, %1, %1;" : "=r"(sq) : "r"(x));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(t) : "r"(sq), "r"(k1), "r"(k0));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(u) : "r"(x), "r"(t));
  asm("tanh.approx.bf16x2 %0, %1;" : "=r"(th) : "r"(u));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(hx) : "r"(x), "r"(half));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(g) : "r"(hx), "r"(th), "r"(hx));
  return g;
}

// Packed bf16x2 arithmetic: one rounding to bf16 per operation.
__device__ __forceinline__ uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// gelu_bf16x2 of 2 h0, 2 h1 given h = x / 2 (the pre-activation carries the
// factor 1/2): u = h (2 k0 + 8 k1 h^2) = x (k0 + k1 x^2), result h + h tanh(u).
// Every rounding sees the same value as in gelu_bf16x2 scaled by a power of
// two, so the results are identical, with one multiply fewer.
__device__ __forceinline__ uint32_t gelu_half_bf16x2(float h0, float h1) {
  uint32_t hx, sq, t, u, th, g;
  asm("cvt.rn.bf16x2.f32 %0, %2, %1;" : "=r"(hx) : "f"(h0), "f"(h1));
  const uint32_t k1 = 0x3E923E92u;   // 8 * bf16x2(0.0356774)
  const uint32_t k0 = 0x3FCC3FCCu;   // 2 * bf16x2(0.7978846)
  asm("mul.rn.bf16x2 %0, %1, %1;" : "=r"(sq) : "r"(hx));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(t) : "r"(sq), "r"(k1), "r"(k0));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(u) : "r"(hx), "r"(t));
  asm("tanh.approx.bf16x2 %0, %1;" : "=r"(th) : "r"(u));
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(g) : "r"(hx), "r"(th), "r"(hx));
  return g;
}

// Packed fp32x2 arithmetic (sm_100): two fp32 lanes per instruction.
struct f2 {
  float x, y;
};
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(r)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)),
        "l"(*reinterpret_cast<uint64_t*>(&c)));
  return *reinterpret_cast<f2*>(&r);
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(r)
      : "l"(*reinterpret_cast<uint64_t*>(&a)), "l"(*reinterpret_cast<uint64_t*>(&b)));
  return *reinterpret_cast<f2*>(&r);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace chm
