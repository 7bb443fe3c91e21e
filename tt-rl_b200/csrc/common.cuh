// Shared device helpers for the sm_100a learner kernels: status codes,
// bounded mbarrier waits, cp.async gathers, TMA, and the tcgen05
// (TMEM allocation, UMMA descriptors, MMA issue, TMEM loads) primitives.
//
// Every wait in this library is bounded: after kWaitTimeoutNs of wall time
// it records an error code in the caller-supplied device status word and the
// kernel unwinds (frees TMEM and returns) instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/ttrl_b200.h"

namespace ttrl {

// One mbarrier wait: polls that each suspend the thread until the phase
// completes or at most kWaitPollNs pass (try_wait's suspend-time hint, which
// the hardware may cut short), so waiting warps sleep instead of spinning on
// the issue slots the working warps need; the global timer, read every 64
// polls, ends the wait after kWaitTimeoutNs.
#ifndef TTRL_WAIT_POLL_NS
#define TTRL_WAIT_POLL_NS 100000
#endif
constexpr uint32_t kWaitPollNs = TTRL_WAIT_POLL_NS;
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Device status codes written into the optional status word.
constexpr int kErrWaitTimeout = 1001;
constexpr int kErrNoValidSlots = 1002;  // a reduction over valid slots found none

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(int* status, int code) {
  if (status != nullptr) atomicExch(status, code);
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}


// Bounded wait on phase `parity` of the barrier. Returns false on timeout.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity,
                                                    uint32_t ns) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_sleep(bar, parity, kWaitPollNs)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_sleep(bar, parity, kWaitPollNs)) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// ------------------------------------------------- programmatic launch

// Every kernel of this library is launched with programmatic stream
// serialization: the next kernel on the stream may start (and do set-up
// that touches no global data) once every CTA of this one has called
// pdl_trigger(). pdl_wait() blocks until the previous kernel has finished
// and its memory is visible; each kernel calls it before its first global
// read or write, so no data race crosses the boundary.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------- composed selects

__device__ __forceinline__ float relu_f(float x) { return x > 0.f ? x : 0.f; }

// clamp(x, lo, hi) as ttrl/engine/ops/select.py:54-63 composes it:
// lifted = relu(x - lo) + lo ; out = hi - relu(hi - lifted). `pass` is the
// derivative (1 strictly inside the band, 0 at or beyond a bound).
__device__ __forceinline__ float clamp_ref(float x, float lo, float hi, float& pass) {
  const float a = __fsub_rn(x, lo);
  const float lifted = __fadd_rn(relu_f(a), lo);
  const float b = __fsub_rn(hi, lifted);
  pass = (a > 0.f && b > 0.f) ? 1.f : 0.f;
  return __fsub_rn(hi, relu_f(b));
}

// ---------------------------------------------------------------- cp.async

// 16-byte global->shared copy; src_bytes == 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  // No "memory" clobber: the destination is read only after cp_async_wait,
  // which carries one, and a clobber here would force the compiler to reload
  // every value it holds from memory after each copy.
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}

// 4-byte global->shared copy; src_bytes == 0 zero-fills the destination.
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes));
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA

// Fetch a tensor map (a kernel parameter) into the TMA unit's descriptor
// cache ahead of its first use; it touches no global data.
__device__ __forceinline__ void prefetch_tensormap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// 2-D tiled TMA load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 4-D TMA load in im2col mode from an NHWC activation: the tensor map's
// pixelsPerColumn pixels starting at window origin (w, h) of image n, walked
// W, then H, then N through the map's bounding box of window origins with its
// traversal strides, each pixel displaced by the filter tap (tap_w, tap_h)
// and contributing channelsPerPixel channels from channel c. Pixels outside
// the tensor read as zeros.
__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const void* tmap, int c, int w,
                                                   int h, int n, uint16_t tap_w, uint16_t tap_h,
                                                   uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], {%7, %8};" ::"r"(dst),
      "l"(tmap), "r"(c), "r"(w), "r"(h), "r"(n), "r"(bar), "h"(tap_w), "h"(tap_h)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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

// Shared-memory matrix descriptor (sm_100 "version 1" format).
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4
//   bits 32-45 stride-dimension byte offset >> 4
//   bits 46-47 version (1 on sm_100)
//   bits 61-63 layout: 2 = SWIZZLE_128B, 1 = SWIZZLE_128B_BASE32B
constexpr uint32_t kLayoutSw128 = 2;
constexpr uint32_t kLayoutSw128Base32 = 1;

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::tf32 with an fp32 accumulator.
//   bits 4-5 D format (1 = f32), 7-9 A format (2 = tf32), 10-12 B format,
//   bit 15 A major (1 = MN), bit 16 B major, bits 17-22 N>>3, bits 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         ((static_cast<uint32_t>(m) >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 32 lanes x 32 bits, 8 consecutive TMEM columns per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Byte offset of element (row, k), k in [0, 32), inside a K-major tile
// stored in the canonical 128-byte-swizzled layout: each row is one
// 128-byte line, rows grouped by 8 into 1024-byte swizzle atoms.
__device__ __forceinline__ uint32_t kmajor_off(int row, int k) {
  return static_cast<uint32_t>(row * 128 + ((((k >> 2) ^ (row & 7)) & 7) << 4) + ((k & 3) << 2));
}

// Byte offset of element (row, k), k in [0, 32), inside an MN-major tile.
// 32-bit MN-major operands use the SWIZZLE_128B_BASE32B layout: a 512-byte
// atom holds 4 k-lines of 32 consecutive rows (128 bytes), with the 32-byte
// granules of each line XOR-swizzled by the line index. The eight 4-line
// k-groups of a 32-wide k-block sit 512 B apart (SBO) and successive
// 32-row groups 4096 B apart (LBO).
__device__ __forceinline__ uint32_t mnmajor_off(int row, int k) {
  const int mn = row & 31;
  const int kr = k & 3;
  return static_cast<uint32_t>((row >> 5) * 4096 + (k >> 2) * 512 + kr * 128 +
                               ((((mn >> 3) ^ kr) & 3) << 5) + ((mn & 7) << 2));
}

// Split x into a tf32-representable high part (low 13 mantissa bits
// cleared) and the exact fp32 remainder.
// x minus its tf32 truncation (the bits a tcgen05 tf32 MMA ignores), exact.
__device__ __forceinline__ float tf32_low(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// x rounded to the nearest tf32 value (ties away from zero), as an fp32
// bit pattern with the low 13 mantissa bits clear. A single-pass tf32 MMA
// would otherwise truncate, a bias that accumulates along the reduction.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

}  // namespace ttrl
