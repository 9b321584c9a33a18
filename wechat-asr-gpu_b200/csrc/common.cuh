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

// Upper bound for any spin-wait on an mbarrier: 2 s of %globaltimer.  A legitimate wait in
// these kernels lasts microseconds; the bound only turns a bug into an error code.
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
// Bounded wait on phase `parity`; false if the 2 s limit passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > WAIT_LIMIT_NS) return false;
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
__device__ __forceinline__ int8_t quant_one(float v, float inv) {
  float q = roundf(__fmul_rn(v, inv));
  q = fminf(127.0f, fmaxf(-127.0f, q));
  return static_cast<int8_t>(q);
}
// GELU of src/model.rs:710-712, evaluated left to right like rustc:
//   ((0.5*x) * (1 + tanh(0.7978846 * (x + ((0.044715*x)*x)*x))))
__device__ __forceinline__ float gelu_ref(float x) {
  float c = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  float u = __fmul_rn(0.7978846f, __fadd_rn(x, c));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(u)));
}
// Epilogue of src/kernels.rs:53: (acc as f32 * xs[i]) * ws + bias (bias 0.0 when absent).
__device__ __forceinline__ float dequant(int32_t acc, float xs, float ws, float bias) {
  return __fadd_rn(__fmul_rn(__fmul_rn(static_cast<float>(acc), xs), ws), bias);
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
