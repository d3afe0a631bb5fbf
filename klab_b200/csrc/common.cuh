// Device helpers shared by every klab_b200 kernel (sm_100a only).
//
// Everything here is hand-written inline PTX or plain CUDA C++: bulk-copy (1-D
// TMA) into shared memory with mbarrier completion, bounded mbarrier waits,
// programmatic dependent launch, packed FP32 FMA (fma.rn.f32x2) and the exact
// widening conversions the projection kernels need. No fast-math, no FTZ: every
// FMA is fma.rn, every add is add.rn, and the one BF16 output rounding is
// cvt.rn.bf16.f32, as in the reference kernels (compressed_kernels.cu:13-24,
// 146-150).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace klab {

// Device status word values. A kernel that gives up a bounded wait records one
// of these (first writer wins) and returns; the host reads and clears the word.
enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusMbarTimeout = 1,     // a bulk copy did not complete within the limit
  kStatusFlagTimeout = 2,     // a peer flag was not raised within the limit
  kStatusBadLength = 3,       // a length read from device memory was out of range
};

// Iteration limit for every spin on an mbarrier or a flag. try_wait suspends for a
// hardware-chosen interval per call, so this bounds a wait to well under a second
// even when no copy ever completes, and the kernel then returns with an error.
constexpr unsigned kSpinLimit = 1u << 22;

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier

__device__ __forceinline__ void mbar_init(unsigned bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(unsigned bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait: true when the phase completed, false after kSpinLimit tries.
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned parity) {
  for (unsigned i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ------------------------------------------------------------------ bulk copy

// 1-D bulk copy global -> shared (no tensor map, this CTA only). dst, src and
// bytes must be multiples of 16; completion is signalled on `bar`.
__device__ __forceinline__ void bulk_g2s(unsigned dst, const void* src, unsigned bytes,
                                         unsigned bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2 (no destination, no completion
// signal). src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before later
// async-proxy (bulk copy) writes to the same shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ peer flags

// System-scope acquire load of a 32-bit flag (written by peers over NVLink).
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// System-scope acquire-release fence: orders this thread's earlier accesses, and
// those it has observed (e.g. its CTA's stores, through a barrier), before its
// later ones for observers on any GPU of the node.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until *flag >= target (monotonic epochs); false on timeout.
__device__ __forceinline__ bool wait_flag_geq(const unsigned* flag, unsigned target) {
  for (unsigned i = 0; i < kSpinLimit; ++i) {
    if (static_cast<int>(ld_acquire_sys(flag) - target) >= 0) return true;
    __nanosleep(64);
  }
  return false;
}

// ------------------------------------------------------------------ PDL

// Wait until the preceding grid in the stream (if launched with programmatic
// stream serialization) has completed and its memory is visible. A no-op for an
// ordinary launch.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ arithmetic

struct f2 {
  float x, y;
};

// d = a * b + c on both halves, each rounded once to nearest even (fma.rn).
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  unsigned long long ra, rb, rc, rd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  f2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(rd));
  return d;
}

// d = a + b on both halves, each rounded once to nearest even (add.rn.f32x2).
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  unsigned long long ra, rb, rd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
  f2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(rd));
  return d;
}

__device__ __forceinline__ float fma_rn(float a, float b, float c) {
  float d;
  asm("fma.rn.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float add_rn(float a, float b) {
  float d;
  asm("add.rn.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

__device__ __forceinline__ float mul_rn(float a, float b) {
  float d;
  asm("mul.rn.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// Butterfly sum over the 32 lanes; every lane ends with the total. The
// association is lanes differing in bit 4 first, then bit 3, ..., bit 0: the same
// tree as the reference's shfl_down reduction (compressed_kernels.cu:26-31) for
// lane 0, because IEEE addition is commutative.
__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int off = 16; off; off >>= 1) v = add_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

__device__ __forceinline__ unsigned short f32_to_bf16_rn(float v) {
  unsigned short b;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(b) : "f"(v));
  return b;
}

// Exact widenings.
__device__ __forceinline__ float bf16lo(unsigned w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(unsigned w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float f16_to_f32(unsigned short h) {
  float f;
  asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h));
  return f;
}
__device__ __forceinline__ float f16lo(unsigned w) { return f16_to_f32(static_cast<unsigned short>(w)); }
__device__ __forceinline__ float f16hi(unsigned w) { return f16_to_f32(static_cast<unsigned short>(w >> 16)); }

// Two E2M1 codes in one byte -> two FP16 values in one word (exact).
__device__ __forceinline__ unsigned e2m1x2_to_f16x2(unsigned byte_value) {
  unsigned d;
  asm("{\n .reg .b8 t;\n cvt.u8.u32 t, %1;\n cvt.rn.f16x2.e2m1x2 %0, t;\n}\n"
      : "=r"(d)
      : "r"(byte_value));
  return d;
}

// Two E4M3 (fn) codes in the low 16 bits -> two FP16 values (exact, NaN kept).
__device__ __forceinline__ unsigned e4m3x2_to_f16x2(unsigned short two_bytes) {
  unsigned d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(two_bytes));
  return d;
}

// ------------------------------------------------------------------ loads

__device__ __forceinline__ uint4 lds128(unsigned addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ unsigned lds32(unsigned addr) {
  unsigned v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ unsigned short lds16(unsigned addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// Read-only global load that does not allocate in L1 (weights, x staging).
__device__ __forceinline__ uint4 ldg128_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// L1-cached read-only load (activations re-read by many warps of one SM).
__device__ __forceinline__ uint4 ldg128_cached(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

}  // namespace klab
