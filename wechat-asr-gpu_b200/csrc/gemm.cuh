// gemm.cuh -- int8 x int8 -> int32 GEMM on the 5th-generation tensor cores (tcgen05,
// kind::i8) with fused epilogues, replacing the reference's cuBLASLt call plus its separate
// epilogue kernels (csrc/wtlgpu.cu:249-380,533-626).
//
//   acc[i][j] = sum_k A[i][k] * B[j][k]        A = activations [M][K], B = weights [N][K]
//
// Both operands are K-major (row-major [rows][K]), exactly the layout of the reference's
// xq buffers and blob weights, so TMA loads them directly with 128-byte swizzle into the
// canonical UMMA K-major layout.  One CTA computes a 128 x BN tile:
//   warp 0      : TMA producer (one elected lane), STAGES-deep smem ring
//   warp 1      : TMEM allocator + MMA issuer (one lane issues tcgen05.mma, M=128, N=BN, K=32)
//   warps 2..5  : epilogue; warp w reads TMEM lanes 32*(w%4).. with tcgen05.ld (thread = row)
// Every spin-wait is bounded (common.cuh); a timeout sets the context's error word.
#pragma once

#include "common.cuh"

namespace wasr {

enum Epi : int {
  EPI_F32 = 0,         // out = (acc*xs)*ws + bias
  EPI_F32_ADD = 1,     // out += (acc*xs)*ws + bias          (residual, src/model.rs:493,496)
  EPI_I32 = 2,         // raw accumulators
  EPI_F32_ROWMAX = 3,  // EPI_F32 + atomic row max of |out|  (first half of wp_gemm_q)
  EPI_GELU_ROWMAX = 4, // out = gelu(...) + row max of |out| (first half of wp_gemm_qg / FF1)
  EPI_ARGMAX = 5,      // per-row (max logit, first index) into packed 64-bit keys
};

struct GemmArgs {
  const int8_t* a;     // [M][K]
  const int8_t* b;     // [N][K]
  int M, N, K;         // N = weight rows multiplied
  int n_store;         // columns written / considered (<= N)
  const float* xs;     // [M] activation row scales
  float ws;            // per-tensor weight scale
  const float* ws_vec; // optional [N] per-output-channel scales (replaces ws)
  const float* bias;   // optional [N]
  float* out;          // fp32 output / residual [M][ldo]
  int ldo;
  int32_t* out_i32;    // EPI_I32 output [M][ldo]
  unsigned* rowmax;    // EPI_*_ROWMAX: float bits of max |v| per row (zeroed by caller)
  unsigned long long* keys;  // EPI_ARGMAX: per-row packed keys (zeroed by caller)
  int* err;            // device error word
  int epi;             // Epi kind
};

template <int EPI>
__device__ __forceinline__ void epi_store_row(const GemmArgs& g, int row, int col0, const int32_t* acc, int ncols,
                                              float& rmax, float& best, uint32_t& bidx) {
  // acc[0..ncols) (ncols <= 32) are columns col0.. of `row`; all are < n_store.
  if constexpr (EPI == EPI_I32) {
    int32_t* o = g.out_i32 + static_cast<int64_t>(row) * g.ldo + col0;
    if (ncols == 32 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4*>(o + j) = make_int4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++)
        if (j < ncols) o[j] = acc[j];
    }
    return;
  } else {
    const float xs = g.xs[row];
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; j++) {
      if (j < ncols) {
        const int col = col0 + j;
        const float ws = g.ws_vec ? __ldg(g.ws_vec + col) : g.ws;
        const float bb = g.bias ? __ldg(g.bias + col) : 0.0f;
        v[j] = dequant(acc[j], xs, ws, bb);
        if constexpr (EPI == EPI_GELU_ROWMAX) v[j] = gelu_ref(v[j]);
        if constexpr (EPI == EPI_F32_ROWMAX || EPI == EPI_GELU_ROWMAX) rmax = fmaxf(rmax, fabsf(v[j]));
        if constexpr (EPI == EPI_ARGMAX) {
          if (v[j] > best) { best = v[j]; bidx = static_cast<uint32_t>(col); }
        }
      }
    }
    if constexpr (EPI == EPI_ARGMAX) return;
    float* o = g.out + static_cast<int64_t>(row) * g.ldo + col0;
    if (ncols == 32 && (reinterpret_cast<uintptr_t>(o) & 15) == 0) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 w = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        if constexpr (EPI == EPI_F32_ADD) {
          const float4 h = *reinterpret_cast<const float4*>(o + j);
          w = make_float4(__fadd_rn(h.x, w.x), __fadd_rn(h.y, w.y), __fadd_rn(h.z, w.z), __fadd_rn(h.w, w.w));
        }
        *reinterpret_cast<float4*>(o + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; j++) {
        if (j < ncols) {
          if constexpr (EPI == EPI_F32_ADD) o[j] = __fadd_rn(o[j], v[j]);
          else o[j] = v[j];
        }
      }
    }
  }
}

template <int EPI>
__device__ __forceinline__ void epi_finish_row(const GemmArgs& g, int row, float rmax, float best, uint32_t bidx) {
  if constexpr (EPI == EPI_F32_ROWMAX || EPI == EPI_GELU_ROWMAX) {
    atomicMax(g.rowmax + row, __float_as_uint(rmax));  // |v| >= 0: uint order == float order
  }
  if constexpr (EPI == EPI_ARGMAX) {
    if (bidx != 0xFFFFFFFFu) atomicMax(g.keys + row, argmax_key(best, bidx));
  }
}

template <int BN>
struct TcCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 128;  // bytes of K per stage = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + (2 * STAGES + 1) * 8 + 16;
};

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_i8_tc(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, GemmArgs g) {
  using Cfg = TcCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * Cfg::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accb = empty + STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accb + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * Cfg::BM;
  const int nk = (g.K + Cfg::BK - 1) / Cfg::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    mbar_init(accb, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tslot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % STAGES, it = kb / STAGES;
        if (kb >= STAGES && !mbar_wait(empty + s, (it - 1) & 1)) {
          atomicExch(g.err, ERR_WAIT_EMPTY);
          *abort_flag = 1;
          break;
        }
        if (*abort_flag) break;
        mbar_arrive_expect_tx(full + s, Cfg::STAGE_BYTES);
        tma_load_2d(sA + s * Cfg::A_BYTES, &tma_a, full + s, kb * Cfg::BK, m0);
        tma_load_2d(sB + s * Cfg::B_BYTES, &tma_b, full + s, kb * Cfg::BK, n0);
        issued++;
      }
      // drain: never leave the CTA while a bulk copy may still write its shared memory
      for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; kb++)
        if (!mbar_wait(full + kb % STAGES, (kb / STAGES) & 1)) atomicExch(g.err, ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(BN);
      for (int kb = 0; kb < nk; kb++) {
        const int s = kb % STAGES, it = kb / STAGES;
        if (!mbar_wait(full + s, it & 1)) {
          atomicExch(g.err, ERR_WAIT_FULL);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES), b0 = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < Cfg::BK / 32; kk++)
          mma_i8(tmem, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), idesc, (kb | kk) != 0);
        mma_commit(empty + s);
      }
      mma_commit(accb);
    }
  } else {
    // epilogue warps 2..5 -> TMEM lane quarter (warp % 4)
    const int q = warp & 3;
    const int row = m0 + q * 32 + lane;
    const bool ok = mbar_wait(accb, 0);
    if (!ok) {
      atomicExch(g.err, ERR_WAIT_ACC);
      *abort_flag = 1;
    }
    __syncwarp();  // lanes may leave the wait loop apart: tcgen05.ld is .sync.aligned
    tc_fence_after();
    float rmax = 0.0f, best = -3.40282347e+38f;
    uint32_t bidx = 0xFFFFFFFFu;
    const bool live = ok && !*abort_flag;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);  // warp-collective
      const int col0 = n0 + c0;
      if (live && row < g.M && col0 < g.n_store) {
        const int nc = min(32, g.n_store - col0);
        epi_store_row<EPI>(g, row, col0, reinterpret_cast<const int32_t*>(r), nc, rmax, best, bidx);
      }
    }
    if (live && row < g.M) epi_finish_row<EPI>(g, row, rmax, best, bidx);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();  // lane 0 ran the MMA loop alone: reconverge before the .sync.aligned dealloc
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// Plain CUDA-core GEMM for shapes the TMA path cannot take (K % 16 != 0 or operands not
// 16-byte aligned).  Same epilogues; exact int32 accumulation.
template <int EPI>
__global__ void __launch_bounds__(256) gemm_i8_simt(GemmArgs g) {
  const int col = blockIdx.x * 32 + (threadIdx.x & 31);
  const int row = blockIdx.y * 8 + (threadIdx.x >> 5);
  if (row >= g.M) return;
  float rmax = 0.0f, best = -3.40282347e+38f;
  uint32_t bidx = 0xFFFFFFFFu;
  if (col < g.n_store) {
    const int8_t* a = g.a + static_cast<int64_t>(row) * g.K;
    const int8_t* b = g.b + static_cast<int64_t>(col) * g.K;
    int32_t acc = 0;
    for (int k = 0; k < g.K; k++) acc += static_cast<int32_t>(a[k]) * static_cast<int32_t>(b[k]);
    epi_store_row<EPI>(g, row, col, &acc, 1, rmax, best, bidx);
  }
  if constexpr (EPI == EPI_F32_ROWMAX || EPI == EPI_GELU_ROWMAX || EPI == EPI_ARGMAX) {
    if (col < g.n_store) epi_finish_row<EPI>(g, row, rmax, best, bidx);
  }
}

// Host side -------------------------------------------------------------------------
// Launch one GEMM; returns 0 or a negative ABI error code.
int gemm_run(const GemmArgs& g, cudaStream_t stream);
// Initialise the tensor-map encoder (driver entry point); false if unavailable.
bool gemm_init();
// Set every kernel's shared-memory attribute on the current device (call outside capture).
bool gemm_prepare();

}  // namespace wasr
