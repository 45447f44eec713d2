// Shared sm_100a device helpers: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (TMEM alloc / MMA / ld / st / commit / fences) and UMMA descriptors.
//
// Everything here is written directly as inline PTX for sm_100a. Every spin on an
// mbarrier is bounded: after DSV32_WAIT_LIMIT_CYCLES of SM clock the waiting thread
// records an error word in device memory, raises the CTA's abort flag and returns
// false, so the kernel winds down instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#define DSV32_DEV __device__ __forceinline__

// ~1 s at 1.9 GHz. Normal waits in these kernels last microseconds.
#ifndef DSV32_WAIT_LIMIT_CYCLES
#define DSV32_WAIT_LIMIT_CYCLES 2000000000LL
#endif

// Error word shared by every kernel of the library (first error wins).
// Layout: (kernel_id << 16) | site. Read and cleared by dsv32_device_status().
__device__ unsigned int g_dsv32_device_error = 0;

// Bound of the pipeline waits (mbar_wait), in SM clock cycles; set per device by
// dsv32_set_wait_limit (failure-detection tests shorten it so that waits run out). Drain waits,
// which let in-flight copies and MMAs land before a CTA exits, keep their own compile-time bound.
__device__ long long g_dsv32_wait_limit = DSV32_WAIT_LIMIT_CYCLES;

enum : unsigned int {
  KID_GEMM = 1,
  KID_INDEX = 2,
};

DSV32_DEV void record_device_error(unsigned int code) {
  atomicCAS(&g_dsv32_device_error, 0u, code);
}

DSV32_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DSV32_DEV uint32_t lane_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(r));
  return r;
}

// ---------------------------------------------------------------- programmatic dependent launch
// Every kernel of the library is launched with programmatic stream serialization: it may start
// while the previous kernel on the stream is still finishing. pdl_wait() blocks until that kernel
// has completed and its memory is visible, so each kernel calls it before its first global memory
// access (only shared-memory / TMEM set-up runs before it). pdl_launch_dependents() then lets the
// next kernel's CTAs be scheduled early; they wait the same way. Without the launch attribute
// both are no-ops.
DSV32_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DSV32_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- mbarrier
DSV32_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

DSV32_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DSV32_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

DSV32_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

DSV32_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of parity `parity` to complete. Returns false if the CTA
// was aborted (by this or another thread) or the limit ran out.
DSV32_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, unsigned int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  const long long limit = g_dsv32_wait_limit;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      record_device_error(code);
      return false;
    }
  }
}

// ---------------------------------------------------------------- thread-block clusters
// The address of the same shared-memory location in CTA `rank` of this CTA's cluster.
DSV32_DEV uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

DSV32_DEV void cluster_store(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}

// Arrive on an mbarrier of another CTA of the cluster; the writes this thread made before it (to
// that CTA's shared memory included) are visible to a cluster-scope acquire of the phase.
DSV32_DEV void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

DSV32_DEV bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Every thread of every CTA of the cluster arrives and waits (release / acquire): at kernel start it
// orders barrier initialisation before any remote access, at the end it keeps every CTA alive until
// the others are done with its shared memory.
DSV32_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Same wait, made warp-uniform: every lane polls, and the warp proceeds only if all
// lanes saw the phase complete. Required before .sync.aligned tcgen05 instructions.
DSV32_DEV bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int* abort_flag, unsigned int code) {
  bool ok = mbar_wait(bar, parity, abort_flag, code);
  return __all_sync(0xffffffffu, ok);
}

// mbar_wait with cluster-scope acquire (for phases completed by another CTA's remote arrive), bounded
// the same way.
DSV32_DEV bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag, unsigned int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const long long t0 = clock64();
  const long long limit = g_dsv32_wait_limit;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      record_device_error(code);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
DSV32_DEV void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

DSV32_DEV void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

DSV32_DEV void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one whole warp; the base address lands in smem.
DSV32_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

DSV32_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

DSV32_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DSV32_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32, issued by a single thread.
DSV32_DEV void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on an mbarrier when all previously issued tcgen05 MMAs of this thread complete.
DSV32_DEV void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Instruction descriptor for kind::i8: signed A/B, s32 accumulator, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_i8(int m, int n) {
  return (2u << 4)                          // D format: S32
         | (1u << 7)                        // A format: signed int8
         | (1u << 10)                       // B format: signed int8
         | (uint32_t(n >> 3) << 17)         // N / 8
         | (uint32_t(m >> 4) << 24);        // M / 16
}

// Shared-memory matrix descriptor for a K-major operand whose rows are `row_bytes`
// long (64 or 128) and stored with the matching TMA swizzle; 8-row core groups are
// 8 * row_bytes apart. The tile base must be aligned to 8 * row_bytes.
DSV32_DEV uint64_t make_sdesc(uint32_t smem_addr, uint32_t row_bytes) {
  const uint64_t swz = (row_bytes == 128) ? 2ull : 4ull;  // SWIZZLE_128B : SWIZZLE_64B
  const uint64_t sbo = (8ull * row_bytes) >> 4;
  return uint64_t((smem_addr >> 4) & 0x3FFFu)  // start address
         | (1ull << 16)                        // leading byte offset (unused for swizzled K-major)
         | (sbo << 32)                         // stride byte offset
         | (1ull << 46)                        // descriptor version (sm_100)
         | (swz << 61);                        // swizzle mode
}

// 32 lanes x 32 columns of 32-bit from TMEM into registers, then wait. The registers are
// threaded through the wait so no use can be scheduled before the data has landed.
DSV32_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// tcgen05.ld of 32 columns without waiting; pair with tmem_wait_ld32 on the same registers.
DSV32_DEV void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

DSV32_DEV void tmem_wait_ld32(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// 16-column variants (the promotion epilogue double-buffers 16-column chunks).
DSV32_DEV void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

DSV32_DEV void tmem_wait_ld16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// relu(x) * 2^-22 for an int32 x with |x| < 2^22, exactly, on the FP32 pipe (no integer op).
// The bit pattern of x >= 0 read as fp32 is the subnormal x * 2^-149; multiplied by 2^127 it is
// x * 2^-22, exact because x has at most 22 significant bits. For -2^22 < x < 0 the pattern is a
// NaN (exponent field all ones), and a saturating multiply returns +0 for a NaN result. The
// saturation bound 1.0 is never reached since x * 2^-22 < 1. Subnormal inputs are kept
// (no .ftz), which the FP32 pipe handles at full rate.
DSV32_DEV float relu_i32_x2m22(uint32_t bits) {
  float r;
  asm("mul.rn.sat.f32 %0, %1, %2;" : "=f"(r) : "f"(__uint_as_float(bits)), "f"(0x1p127f));
  return r;
}

// 16-byte asynchronous copy global -> shared (no registers held while in flight); src_bytes = 0
// zero-fills the destination without reading. Completion: cp_async_wait_all() by the issuing thread.
DSV32_DEV void cp_async16(uint32_t smem_dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_dst), "l"(src), "r"(src_bytes) : "memory");
}
DSV32_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
DSV32_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Width-generic forms of the pipelined TMEM reads (16 or 32 columns).
template <int W>
DSV32_DEV void tmem_ld_async(uint32_t taddr, uint32_t (&r)[W]) {
  if constexpr (W == 32) tmem_ld32_async(taddr, r); else tmem_ld16_async(taddr, r);
}
template <int W>
DSV32_DEV void tmem_wait_ld(uint32_t (&r)[W]) {
  if constexpr (W == 32) tmem_wait_ld32(r); else tmem_wait_ld16(r);
}

// Register re-balancing between warpgroups (all 4 warps of a warpgroup execute it).
template <uint32_t N>
DSV32_DEV void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <uint32_t N>
DSV32_DEV void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

// Named barrier over a subset of warps (ids 1..15; 0 is __syncthreads).
DSV32_DEV void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
