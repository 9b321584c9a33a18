// common.cuh -- shared device helpers for libwasr_gpu.so (sm_100a only).
//
// Numerics: wherever the reference CPU path (src/kernels.rs, src/model.rs) fixes an
// evaluation order, device code uses the explicitly rounded intrinsics (__fmul_rn,
// __fadd_rn, __fdiv_rn, __fsqrt_rn), which nvcc never contracts into FMA, so results are
// bit-identical to the CPU.  Free-order code (reductions the CPU does not pin) may use FMA.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "libwasr_gpu targets sm_100a only"
#endif

namespace wasr {

constexpr int D = 512, HEADS = 8, HD = 64, FF = 2048, DIM = 40, C1 = 32, C2 = 64, C3 = 192;
constexpr int W2 = 41, FLAT = 3840, K2 = C1 * 49, K3 = C2 * 9;

// Device error codes written to a context's error word when a bounded wait gives up.
enum : int { ERR_WAIT_FULL = 1, ERR_WAIT_EMPTY = 2, ERR_WAIT_ACC = 3 };

// Default upper bound for any spin-wait on an mbarrier: 2 s of %globaltimer.  A legitimate
// wait in these kernels lasts microseconds; the bound only turns a bug into an error code.
// Kernels take the bound as an argument (0 = this default), so a test can shorten it.
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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
// Bounded wait on phase `parity`; false once limit_ns of %globaltimer passed without it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = WAIT_LIMIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------- TMA (no multicast)
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2-D tiled load of one box into shared memory, completing on `bar` (transaction bytes).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Prefetch of one 2-D box into L2 (no shared memory, no completion: a hint).  x must satisfy
// the same 16-byte rule as a load.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* m, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(m)),
               "r"(x), "r"(y)
               : "memory");
}

// 2-D tiled store of one box from shared memory (bulk-group completion).  The box is clipped
// to the tensor's bounds, so rows / columns past the end are never written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N of this thread's committed bulk groups still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// wait until all of this thread's committed bulk groups have completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// order this thread's generic-proxy shared-memory accesses before later async-proxy (TMA) ones
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- cp.async (global -> shared)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 x int8 -> int32, issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once all previously issued tcgen05.mma of this thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// The same load split in two: tmem_ld32_issue starts it, tmem_ld32_wait (tcgen05.wait::ld, which
// waits for every earlier tcgen05.ld of the thread) completes it.  The wait names the 32
// registers as read-write operands, so no use of them can move above it; work placed between the
// two overlaps the load.
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tmem_ld32_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Store of 32 lanes x 32 consecutive 32-bit columns (thread i of the warp writes row lane base +
// i); tmem_st_wait (tcgen05.wait::st) waits for every earlier tcgen05.st of the thread.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp receives row (lane base + i).
// The wait is inside the same asm block so no use of the registers can move above it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// UMMA shared-memory descriptor for a K-major operand tile written by TMA with 128-byte
// swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart (SBO), version 1 (sm_100),
// layout type 2 = SWIZZLE_128B.  The leading-byte offset is unused for swizzled K-major.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::i8: D = s32, A = B = signed int8, both K-major,
// M = 128, N = n (multiple of 16, <= 256).
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}

// ---------------------------------------------------------------- numerics
// Per-row dynamic quantisation step of src/kernels.rs:17-21: s = m/127 (1 if m == 0),
// inv = 1/s, q = round_half_away(v * inv) clamped to [-127, 127].
__device__ __forceinline__ float quant_scale(float m) { return m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f; }
__device__ __forceinline__ float quant_inv(float s) { return __fdiv_rn(1.0f, s); }
// The clamp and cast follow Rust's `.clamp(-127.0, 127.0) as i8`: NaN gives 0 and +-inf +-127.
// The float -> int conversion (cvt.rzi: saturating, NaN to 0) comes first and the clamp is
// then an integer one; for the integral values round() gives it equals the float clamp.
__device__ __forceinline__ int8_t quant_one(float v, float inv) {
  const int q = __float2int_rz(roundf(__fmul_rn(v, inv)));
  return static_cast<int8_t>(min(127, max(-127, q)));
}
// ---------------------------------------------------------------- libm restatements
// The reference CPU path calls the platform libm: Rust's f32::tanh / f32::exp are glibc's
// tanhf / expf (glibc 2.39 on this image).  CUDA's tanhf / expf differ from those in the last
// place for a few percent of inputs, and over 40 layers such one-ulp differences flip int8
// roundings that the random network then amplifies.  So the kernels evaluate the same
// published algorithms glibc uses, with every operation explicitly rounded:
//   tanhf: the fdlibm algorithm (tanh via expm1: 1 - 2/(expm1(2|x|)+2) for |x| >= 1,
//          -t/(t+2) with t = expm1(-2|x|) below, +-1 beyond 22);
//   expm1f: fdlibm's argument reduction by ln2 (hi/lo split) and its rational correction
//          with the five-term polynomial in x^2/2;
//   expf: the table-driven double-precision method (x*32/ln2 = k + r, 2^(k/32) from a 32-entry
//          table of 2^(i/32), cubic polynomial in r).
// Exhaustive comparison against glibc on every float input: tanhf identical for all
// 4,278,190,082 non-NaN inputs; expf identical for all inputs except two, which are special-
// cased below with glibc's values.
//
// Upstream sources of the restated algorithms and their constants, with their notices:
// * tanhf_ref / expm1f_ref follow fdlibm's s_tanh.c / s_expm1.c as converted to float
//   (s_tanhf.c / s_expm1f.c, conversion by Ian Lance Taylor, Cygnus Support), the versions
//   glibc ships in sysdeps/ieee754/flt-32:
//     Copyright (C) 1993 by Sun Microsystems, Inc. All rights reserved.
//     Developed at SunPro, a Sun Microsystems, Inc. business.
//     Permission to use, copy, modify, and distribute this software is freely granted,
//     provided that this notice is preserved.
// * expf_body follows the expf of Arm's optimized-routines (math/expf.c, its 2^(i/32) table
//   and polynomial), which glibc ships as sysdeps/ieee754/flt-32/e_expf.c:
//     Copyright (c) 2017-2018, Arm Limited.  SPDX-License-Identifier: MIT.
//     Permission is hereby granted, free of charge, to any person obtaining a copy of this
//     software and associated documentation files (the "Software"), to deal in the Software
//     without restriction, including without limitation the rights to use, copy, modify,
//     merge, publish, distribute, sublicense, and/or sell copies of the Software, and to
//     permit persons to whom the Software is furnished to do so, subject to the following
//     conditions: The above copyright notice and this permission notice shall be included in
//     all copies or substantial portions of the Software.  THE SOFTWARE IS PROVIDED "AS IS",
//     WITHOUT WARRANTY OF ANY KIND, EXPRESS OR IMPLIED, INCLUDING BUT NOT LIMITED TO THE
//     WARRANTIES OF MERCHANTABILITY, FITNESS FOR A PARTICULAR PURPOSE AND NONINFRINGEMENT. IN
//     NO EVENT SHALL THE AUTHORS OR COPYRIGHT HOLDERS BE LIABLE FOR ANY CLAIM, DAMAGES OR OTHER
//     LIABILITY, WHETHER IN AN ACTION OF CONTRACT, TORT OR OTHERWISE, ARISING FROM, OUT OF OR
//     IN CONNECTION WITH THE SOFTWARE OR THE USE OR OTHER DEALINGS IN THE SOFTWARE.
__device__ __forceinline__ float f_from_bits(uint32_t u) { return __uint_as_float(u); }

// expm1f, branch-free: every path of the fdlibm algorithm shares the argument reduction
// (k = 0, +-1 or round(x/ln2); hi = x - k*ln2_hi, lo = k*ln2_lo) and the rational core, and
// differs only in a few-operation reconstruction; all reconstructions are evaluated and the
// right one selected, so the lanes of a warp never diverge.  Bit-identical to glibc's expm1f
// on |x| < 88, as the branch-free tanhf built on it is to glibc's tanhf on every float input
// (exhaustive host comparison).
__device__ __forceinline__ float expm1f_ref(float x) {
  const float ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f, invln2 = 1.4426950216e+00f;
  const float Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f, Q4 = 4.0082177293e-06f,
              Q5 = -2.0109921195e-07f;
  uint32_t hx = __float_as_uint(x);
  const uint32_t xsb = hx >> 31;
  hx &= 0x7fffffffu;
  const int kgen = static_cast<int>(__fadd_rn(__fmul_rn(invln2, x), xsb ? -0.5f : 0.5f));
  const int k = hx > 0x3eb17218u ? (hx < 0x3F851592u ? (xsb ? -1 : 1) : kgen) : 0;
  const float tk = static_cast<float>(k);
  const float hi = __fsub_rn(x, __fmul_rn(tk, ln2_hi)), lo = __fmul_rn(tk, ln2_lo);
  const float xr = __fsub_rn(hi, lo);
  const float c = __fsub_rn(__fsub_rn(hi, xr), lo);
  const float hfx = __fmul_rn(0.5f, xr);
  const float hxs = __fmul_rn(xr, hfx);
  float r1 = __fmul_rn(hxs, Q5);
  r1 = __fmul_rn(hxs, __fadd_rn(Q4, r1));
  r1 = __fmul_rn(hxs, __fadd_rn(Q3, r1));
  r1 = __fmul_rn(hxs, __fadd_rn(Q2, r1));
  r1 = __fadd_rn(1.0f, __fmul_rn(hxs, __fadd_rn(Q1, r1)));
  const float t = __fsub_rn(3.0f, __fmul_rn(r1, hfx));
  const float e = __fmul_rn(hxs, __fdiv_rn(__fsub_rn(r1, t), __fsub_rn(6.0f, __fmul_rn(xr, t))));
  const float res0 = __fsub_rn(xr, __fsub_rn(__fmul_rn(xr, e), hxs));
  const float e2 = __fsub_rn(__fsub_rn(__fmul_rn(xr, __fsub_rn(e, c)), c), hxs);
  const float resm1 = __fsub_rn(__fmul_rn(0.5f, __fsub_rn(xr, e2)), 0.5f);
  const float resp1 = xr < -0.25f ? __fmul_rn(-2.0f, __fsub_rn(e2, __fadd_rn(xr, 0.5f)))
                                  : __fadd_rn(1.0f, __fmul_rn(2.0f, __fsub_rn(xr, e2)));
  const uint32_t kexp = static_cast<uint32_t>(k) << 23;
  const float yA = __fsub_rn(1.0f, __fsub_rn(e2, xr));
  const float resA = __fsub_rn(f_from_bits(__float_as_uint(yA) + kexp), 1.0f);
  const int kb = k < 0 ? 0 : (k > 31 ? 31 : k);
  const float yB = __fsub_rn(f_from_bits(0x3f800000u - (0x1000000u >> kb)), __fsub_rn(e2, xr));
  const float resB = f_from_bits(__float_as_uint(yB) + kexp);
  const int kc = k < 0 ? 0 : (k > 127 ? 127 : k);
  float yC = __fsub_rn(xr, __fadd_rn(e2, f_from_bits(static_cast<uint32_t>(0x7f - kc) << 23)));
  yC = __fadd_rn(yC, 1.0f);
  const float resC = f_from_bits(__float_as_uint(yC) + kexp);
  float r = k == 0 ? res0 : k == -1 ? resm1 : k == 1 ? resp1 : (k <= -2 || k > 56) ? resA : k < 23 ? resB : resC;
  r = (hx >= 0x4195b844u && xsb) ? -1.0f : r;               // x < -27 ln2
  r = (hx <= 0x3eb17218u && hx < 0x33000000u) ? x : r;      // |x| < 2^-25
  return r;
}

// tanhf, branch-free: tanh(|x|) = 1 - 2/(expm1(2|x|)+2) for |x| >= 1, -t/(t+2) with
// t = expm1(-2|x|) below 1, 1 - 1e-30 from 22 on; odd symmetry; the tiny / zero / non-finite
// cases of the reference algorithm as selects.  The expm1 is fdlibm's, specialised to the two
// argument ranges tanh gives it: y in (-2, 0] (k = 0, -1, -2 or -3) and y in [2, 44) (k >= 3).
// Hence no k = 1 reconstruction; the k <= -2 and 3 <= k < 23 reconstructions share
// y' = C - (e2 - x) with C = 1 or 1 - 2^-k, and all three non-trivial ones share the final
// exponent add.  For k > 56 fdlibm's own reconstruction differs, but there t > 2^56 and tanh
// rounds to 1 either way.  Identical to glibc's tanhf for all 4,278,190,082 non-NaN floats
// (exhaustive host comparison of the same operation sequence).
// a / b rounded to nearest for the divisions inside tanhf_ref, whose divisors are normal and
// finite wherever the result is used: the reciprocal from the hardware approximation
// (rcp.approx) refined by one Newton-Raphson step, then Markstein's correction of the quotient
// (q = RN(a*y), r = fma(-q, b, a) exact, RN(q + r*y)), the published method of P. Markstein,
// IBM J. Res. Dev. 34(1), 1990, and Muller et al., Handbook of Floating-Point Arithmetic.
// tanhf_ref with it equals tanhf_ref with __fdiv_rn on all 2^32 inputs (checked on the GPU).
__device__ __forceinline__ float div_nr(float a, float b) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(b));
  y = __fmaf_rn(__fmaf_rn(-b, y, 1.0f), y, y);
  const float q = __fmul_rn(a, y);
  return __fmaf_rn(__fmaf_rn(-q, b, a), y, q);
}

__device__ __forceinline__ float tanhf_ref(float x) {
  const float ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f, invln2 = 1.4426950216e+00f;
  const float Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f, Q4 = 4.0082177293e-06f,
              Q5 = -2.0109921195e-07f;
  const uint32_t jx = __float_as_uint(x), ix = jx & 0x7fffffffu;
  const float ax = fabsf(x);
  const bool ge1 = ix >= 0x3f800000u;
  const float y = __fmul_rn(ge1 ? 2.0f : -2.0f, ax);  // exact
  const uint32_t hy = __float_as_uint(y) & 0x7fffffffu;
  const int kgen = static_cast<int>(__fadd_rn(__fmul_rn(invln2, y), ge1 ? 0.5f : -0.5f));
  const int k = ge1 ? kgen : (hy <= 0x3eb17218u ? 0 : (hy < 0x3F851592u ? -1 : kgen));
  const float tk = static_cast<float>(k);
  const float hi = __fsub_rn(y, __fmul_rn(tk, ln2_hi)), lo = __fmul_rn(tk, ln2_lo);
  const float xr = __fsub_rn(hi, lo);
  const float c = __fsub_rn(__fsub_rn(hi, xr), lo);
  const float hfx = __fmul_rn(0.5f, xr);
  const float hxs = __fmul_rn(xr, hfx);
  float r1 = __fmul_rn(hxs, Q5);
  r1 = __fmul_rn(hxs, __fadd_rn(Q4, r1));
  r1 = __fmul_rn(hxs, __fadd_rn(Q3, r1));
  r1 = __fmul_rn(hxs, __fadd_rn(Q2, r1));
  r1 = __fadd_rn(1.0f, __fmul_rn(hxs, __fadd_rn(Q1, r1)));
  const float t = __fsub_rn(3.0f, __fmul_rn(r1, hfx));
  const float e = __fmul_rn(hxs, div_nr(__fsub_rn(r1, t), __fsub_rn(6.0f, __fmul_rn(xr, t))));
  const float res0 = __fsub_rn(xr, __fsub_rn(__fmul_rn(xr, e), hxs));
  const float e2 = __fsub_rn(__fsub_rn(__fmul_rn(xr, __fsub_rn(e, c)), c), hxs);
  const float resm1 = __fsub_rn(__fmul_rn(0.5f, __fsub_rn(xr, e2)), 0.5f);
  const float two_mk = f_from_bits(static_cast<uint32_t>(0x7f - k) << 23);  // 2^-k, k in [-3, 63]
  const float cab = k < 0 ? 1.0f : __fsub_rn(1.0f, two_mk);
  const float yab = __fsub_rn(cab, __fsub_rn(e2, xr));
  const float yc = __fadd_rn(__fsub_rn(xr, __fadd_rn(e2, two_mk)), 1.0f);
  const float ysel = k < 23 ? yab : yc;
  float rr = f_from_bits(__float_as_uint(ysel) + (static_cast<uint32_t>(k) << 23));
  rr = k < 0 ? __fsub_rn(rr, 1.0f) : rr;
  float em = k == 0 ? res0 : (k == -1 ? resm1 : rr);
  em = (!ge1 && hy < 0x33000000u) ? y : em;  // |y| < 2^-25: expm1(y) = y
  const float q = div_nr(ge1 ? 2.0f : -em, __fadd_rn(em, 2.0f));
  float z = ge1 ? __fsub_rn(1.0f, q) : q;
  z = ix >= 0x41b00000u ? __fsub_rn(1.0f, 1.0e-30f) : z;
  float r = (jx >> 31) ? -z : z;
  r = ix < 0x24000000u ? __fmul_rn(x, __fadd_rn(1.0f, x)) : r;
  r = ix == 0 ? x : r;
  if (ix >= 0x7f800000u)  // non-finite input: 1/x -+ 1 as in the reference
    r = (jx >> 31) ? __fsub_rn(__fdiv_rn(1.0f, x), 1.0f) : __fadd_rn(__fdiv_rn(1.0f, x), 1.0f);
  return r;
}

__constant__ static const unsigned long long kExp2Tab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

// tab[i] above = bits(2^(i/32)) - (i << 47): adding k << 47 to tab[k % 32] yields 2^(k/32).
// `lookup(i)` returns tab[i]: from constant memory (expf_ref) or from a shared-memory copy
// (expf_ref_smem; indexed constant loads serialise when the lanes of a warp differ).
// Branch-free: the main path runs for every input and the special ranges are selected after
// it, so several calls in a row can overlap (the double-precision chain is ~230 cycles long).
template <typename Lookup>
__device__ __forceinline__ float expf_body(float x, Lookup lookup) {
  const uint32_t ux = __float_as_uint(x);
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
  const double shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32768.0;  // cubic coefficients of 2^(r/32), r in [-1/2, 1/2]
  const double c1 = 0x1.ebfce50fac4f3p-3 / 1024.0;
  const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double z = __dmul_rn(inv_ln2_n, static_cast<double>(x));
  double kd = __dadd_rn(z, shift);
  const unsigned long long ki = static_cast<unsigned long long>(__double_as_longlong(kd));
  kd = __dsub_rn(kd, shift);
  const double r = __dsub_rn(z, kd);
  const unsigned long long t = lookup(static_cast<int>(ki & 31)) + (ki << 47);
  const double s = __longlong_as_double(static_cast<long long>(t));
  const double zz = __dadd_rn(__dmul_rn(c0, r), c1);
  const double r2 = __dmul_rn(r, r);
  double y = __dadd_rn(__dmul_rn(c2, r), 1.0);
  y = __dadd_rn(__dmul_rn(zz, r2), y);
  y = __dmul_rn(y, s);
  float res = __double2float_rn(y);
  const uint32_t abstop = (ux >> 20) & 0x7ffu;
  if (abstop >= (0x42b00000u >> 20)) {  // |x| >= 88 or non-finite (the main path result is
    // kept for x in [88, 88.72] and [-103.97, -88], as in the reference algorithm)
    res = x < -103.97207641601562f ? 0.0f : res;
    res = x > 88.72283172607421875f ? __int_as_float(0x7f800000) : res;
    res = abstop >= (0x7f800000u >> 20) ? __fadd_rn(x, x) : res;
    res = ux == 0xff800000u ? 0.0f : res;
  }
  res = ux == 0x4202422fu ? f_from_bits(0x56fc9f1cu) : res;  // the two inputs where glibc's result
  res = ux == 0xc27c65d9u ? f_from_bits(0x11fa2993u) : res;  // is the other float neighbour
  return res;
}
__device__ __forceinline__ float expf_ref(float x) {
  return expf_body(x, [](int i) { return kExp2Tab[i]; });
}
// tab: a shared-memory copy of kExp2Tab
__device__ __forceinline__ float expf_ref_smem(float x, const unsigned long long* tab) {
  return expf_body(x, [tab](int i) { return tab[i]; });
}

// GELU of src/model.rs:710-712, evaluated left to right like rustc:
//   ((0.5*x) * (1 + tanh(0.7978846 * (x + ((0.044715*x)*x)*x))))
__device__ __forceinline__ float gelu_ref(float x) {
  float c = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  float u = __fmul_rn(0.7978846f, __fadd_rn(x, c));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf_ref(u)));
}
// ---- the same tanhf / GELU for two independent elements: every multiply is one packed
// multiply of the pair (mul.rn.f32x2); every add and divide, and every subtract with a product
// as an operand, stays a scalar rounded operation per element (so no multiply can be contracted
// into an add); a subtract of two scalar results is one packed sub.rn.f32x2; the integer /
// select logic runs per element.  Identical results to tanhf_ref / gelu_ref element by element.
__device__ __forceinline__ float2 pmul2(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"((static_cast<unsigned long long>(__float_as_uint(a.y)) << 32) |
                                                 __float_as_uint(a.x)),
      "l"((static_cast<unsigned long long>(__float_as_uint(b.y)) << 32) | __float_as_uint(b.x)));
  return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}
__device__ __forceinline__ float2 f2c(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 sadd2(float2 a, float2 b) { return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)); }
__device__ __forceinline__ float2 ssub2(float2 a, float2 b) { return make_float2(__fsub_rn(a.x, b.x), __fsub_rn(a.y, b.y)); }
__device__ __forceinline__ float2 sdiv2(float2 a, float2 b) { return make_float2(div_nr(a.x, b.x), div_nr(a.y, b.y)); }
// packed subtract, used only where neither operand comes straight from a packed multiply
__device__ __forceinline__ float2 psub2(float2 a, float2 b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"((static_cast<unsigned long long>(__float_as_uint(a.y)) << 32) |
                                                 __float_as_uint(a.x)),
      "l"((static_cast<unsigned long long>(__float_as_uint(b.y)) << 32) | __float_as_uint(b.x)));
  return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}

// per-element part of tanhf_ref after the shared reductions: reconstruction, tanh, specials
__device__ __forceinline__ float tanh_tail(float x, int k, bool ge1, uint32_t hy, float y, float xr, float e2, float res0,
                                           float resm1) {
  const uint32_t jx = __float_as_uint(x), ix = jx & 0x7fffffffu;
  const float two_mk = f_from_bits(static_cast<uint32_t>(0x7f - k) << 23);
  const float cab = k < 0 ? 1.0f : __fsub_rn(1.0f, two_mk);
  const float yab = __fsub_rn(cab, __fsub_rn(e2, xr));
  const float yc = __fadd_rn(__fsub_rn(xr, __fadd_rn(e2, two_mk)), 1.0f);
  const float ysel = k < 23 ? yab : yc;
  float rr = f_from_bits(__float_as_uint(ysel) + (static_cast<uint32_t>(k) << 23));
  rr = k < 0 ? __fsub_rn(rr, 1.0f) : rr;
  float em = k == 0 ? res0 : (k == -1 ? resm1 : rr);
  em = (!ge1 && hy < 0x33000000u) ? y : em;
  const float q = div_nr(ge1 ? 2.0f : -em, __fadd_rn(em, 2.0f));
  float z = ge1 ? __fsub_rn(1.0f, q) : q;
  z = ix >= 0x41b00000u ? __fsub_rn(1.0f, 1.0e-30f) : z;
  float r = (jx >> 31) ? -z : z;
  r = ix < 0x24000000u ? __fmul_rn(x, __fadd_rn(1.0f, x)) : r;
  r = ix == 0 ? x : r;
  if (ix >= 0x7f800000u)
    r = (jx >> 31) ? __fsub_rn(__fdiv_rn(1.0f, x), 1.0f) : __fadd_rn(__fdiv_rn(1.0f, x), 1.0f);
  return r;
}

__device__ __forceinline__ float2 tanhf_ref2(float2 x) {
  const float ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f, invln2 = 1.4426950216e+00f;
  const float Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f, Q4 = 4.0082177293e-06f,
              Q5 = -2.0109921195e-07f;
  const uint32_t ia = __float_as_uint(x.x) & 0x7fffffffu, ib = __float_as_uint(x.y) & 0x7fffffffu;
  const bool ga = ia >= 0x3f800000u, gb = ib >= 0x3f800000u;
  const float2 y = pmul2(make_float2(ga ? 2.0f : -2.0f, gb ? 2.0f : -2.0f), make_float2(fabsf(x.x), fabsf(x.y)));
  const uint32_t hya = __float_as_uint(y.x) & 0x7fffffffu, hyb = __float_as_uint(y.y) & 0x7fffffffu;
  const float2 iy = pmul2(f2c(invln2), y);
  const int kga = static_cast<int>(__fadd_rn(iy.x, ga ? 0.5f : -0.5f));
  const int kgb = static_cast<int>(__fadd_rn(iy.y, gb ? 0.5f : -0.5f));
  const int ka = ga ? kga : (hya <= 0x3eb17218u ? 0 : (hya < 0x3F851592u ? -1 : kga));
  const int kb = gb ? kgb : (hyb <= 0x3eb17218u ? 0 : (hyb < 0x3F851592u ? -1 : kgb));
  const float2 tk = make_float2(static_cast<float>(ka), static_cast<float>(kb));
  const float2 hi = ssub2(y, pmul2(tk, f2c(ln2_hi))), lo = pmul2(tk, f2c(ln2_lo));
  const float2 xr = ssub2(hi, lo);
  const float2 c = ssub2(psub2(hi, xr), lo);
  const float2 hfx = pmul2(f2c(0.5f), xr);
  const float2 hxs = pmul2(xr, hfx);
  float2 r1 = pmul2(hxs, f2c(Q5));
  r1 = pmul2(hxs, sadd2(f2c(Q4), r1));
  r1 = pmul2(hxs, sadd2(f2c(Q3), r1));
  r1 = pmul2(hxs, sadd2(f2c(Q2), r1));
  r1 = sadd2(f2c(1.0f), pmul2(hxs, sadd2(f2c(Q1), r1)));
  const float2 t = ssub2(f2c(3.0f), pmul2(r1, hfx));
  const float2 e = pmul2(hxs, sdiv2(psub2(r1, t), ssub2(f2c(6.0f), pmul2(xr, t))));
  const float2 res0 = psub2(xr, ssub2(pmul2(xr, e), hxs));
  const float2 e2 = ssub2(ssub2(pmul2(xr, ssub2(e, c)), c), hxs);
  const float2 resm1 = ssub2(pmul2(f2c(0.5f), psub2(xr, e2)), f2c(0.5f));
  return make_float2(tanh_tail(x.x, ka, ga, hya, y.x, xr.x, e2.x, res0.x, resm1.x),
                     tanh_tail(x.y, kb, gb, hyb, y.y, xr.y, e2.y, res0.y, resm1.y));
}

__device__ __forceinline__ float2 gelu_ref2(float2 x) {
  const float2 c = pmul2(pmul2(pmul2(f2c(0.044715f), x), x), x);
  const float2 u = pmul2(f2c(0.7978846f), sadd2(x, c));
  return pmul2(pmul2(f2c(0.5f), x), sadd2(f2c(1.0f), tanhf_ref2(u)));
}

// a / b rounded to nearest for a in [0, 1] and b in [1, 2^24) (a softmax numerator and row
// sum), given yb = __frcp_rn(b): Markstein's correction (P. Markstein, IBM J. Res. Dev. 34(1),
// 1990, "Computation of elementary functions on the IBM RISC System/6000 processor"): with yb
// the correctly rounded reciprocal and q within an ulp of a/b, r = a - b*q is exact (one fma)
// and RN(q + r*yb) is the correctly rounded quotient.  Numerators below 2^-80 (where q or r
// could underflow) need the full division: div_unit_fast leaves them to the caller
// (div_unit_tiny), which tests for them once per warp so the common case has no division.
__device__ __forceinline__ float div_unit_fast(float a, float b, float yb) {
  const float q = __fmul_rn(a, yb);
  const float r = __fmaf_rn(-q, b, a);
  return __fmaf_rn(r, yb, q);
}
__device__ __forceinline__ bool div_unit_tiny(float a) { return a < 0x1p-80f; }
__device__ __forceinline__ float div_unit_rn(float a, float b, float yb) {
  return div_unit_tiny(a) ? __fdiv_rn(a, b) : div_unit_fast(a, b, yb);
}

// Epilogue of src/kernels.rs:53: (acc as f32 * xs[i]) * ws + bias (bias 0.0 when absent).
__device__ __forceinline__ float dequant(int32_t acc, float xs, float ws, float bias) {
  return __fadd_rn(__fmul_rn(__fmul_rn(static_cast<float>(acc), xs), ws), bias);
}

// Packed FP32x2 multiply / add with round-to-nearest per component (Blackwell).  Each is exact
// on its own, but a packed multiply feeding a packed add is contracted into a packed fused
// multiply-add by the code generator (measured: results equal fmaf's), so exact sequences pair
// a packed multiply with scalar __fadd_rn adds, or scalar __fmul_rn products with a packed add.
__device__ __forceinline__ unsigned long long f2_bits(float2 a) {
  return (static_cast<unsigned long long>(__float_as_uint(a.y)) << 32) | __float_as_uint(a.x);
}
__device__ __forceinline__ float2 bits_f2(unsigned long long u) {
  return make_float2(__uint_as_float(static_cast<uint32_t>(u)), __uint_as_float(static_cast<uint32_t>(u >> 32)));
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(r);
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(r);
}

// ---- certified approximate GELU.  The GELU output is consumed only by its row's int8
// quantisation (src/model.rs:495-496: quant(gelu(f))), so the quantised row equals the exact
// one whenever (a) the row maximum is taken from exact values and (b) no element's scaled value
// lies within the approximation's error of a rounding boundary.  gelu_fast2 evaluates
// 0.5 x (1 + tanh u) = x / (1 + e^(-2u)), u = 0.7978846 (x + 0.044715 x^3), as
// x * rcp(1 + 2^(x (k1 + k3 x^2))) with k1 = -2 * 0.7978846 / ln 2, k3 = 0.044715 k1, from the
// hardware exp2 and reciprocal approximations.  For every float x with gelu_ref(x) finite:
//     gelu_fast(x) finite  =>  |gelu_fast(x) - gelu_ref(x)| <= GELU_CERT_A + GELU_CERT_B |gelu_fast(x)|
//     gelu_fast(x) non-finite is allowed (the kernel then runs the row exactly),
// and gelu_fast(x) is non-finite wherever gelu_ref(x) is.  Checked on all 2^32 inputs on the
// GPU (wasr_gelu_cert_scan).
constexpr float GELU_CERT_A = 0x1p-23f;
constexpr float GELU_CERT_B = 0x1p-21f;
// |gelu_ref(x)| <= GELU_NEG_MAX for every x < 0, and gelu_ref is non-decreasing on [0, inf]
// (both checked on every float by wasr_gelu_cert_scan)
constexpr float GELU_NEG_MAX = 0.171f;
// fma(v, inv, RINT_MAGIC) rounds v * inv to the nearest integer n (ties to even), held in the
// low mantissa bits for |v * inv| < 2^22: the result's low byte is n as an int8
constexpr float RINT_MAGIC = 12582912.0f;  // 1.5 * 2^23
// packed fused multiply-add, one rounding per element
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(r);
}
__device__ __forceinline__ float2 gelu_fast2(float2 x) {
  const float2 x2 = pmul2(x, x);
  const float2 a = pmul2(fma2_rn(x2, f2c(-0x1.a5a7d0p-4f), f2c(-0x1.26aec4p+1f)), x);  // -2u / ln 2
  float ex, ey, rx, ry;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(ex) : "f"(a.x));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(ey) : "f"(a.y));
  const float2 d = add2_rn(f2c(1.0f), make_float2(ex, ey));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rx) : "f"(d.x));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(ry) : "f"(d.y));
  return pmul2(x, make_float2(rx, ry));
}

// Order-preserving map of a float to uint32 (for packed argmax keys).
__device__ __forceinline__ uint32_t float_order(float v) {
  uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Argmax key: larger value wins, equal values prefer the lower index (first max wins).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  return (static_cast<unsigned long long>(float_order(v)) << 32) | (0xFFFFFFFFu - idx);
}

}  // namespace wasr
