// gemm_gq.cuh -- the feed-forward up-projection, its GELU and the per-row int8 quantisation of
// the GELU output in one tcgen05 kernel (src/model.rs:495-496: f1 + bias, gelu, then quant of
// src/kernels.rs:11-25), so that the [M][FF] fp32 activations never reach HBM.
//
// The row's int8 values and scale must equal quant(gelu(x)) of the reference, where
// x = dequant(acc) is the f1 GEMM's exact fp32 output.  The kernel uses the certified GELU
// approximation of the standalone GELU kernel (gelu_fast2, bound GELU_CERT_A + GELU_CERT_B |g~|,
// checked on every float) and the same row logic:
//  * the exact row maximum is M = gelu_ref(max x) whenever that is >= GELU_NEG_MAX (gelu_ref is
//    non-decreasing on [0, inf] and at most GELU_NEG_MAX in magnitude below 0);
//  * an element whose scaled approximation lies within the bound of a rounding boundary is
//    quantised again from gelu_ref(x), x being exact in the epilogue.
// A row needs max x before any element can be quantised, and a 128 x 2048 fp32 block does not
// fit in tensor memory, so a CTA makes two passes over its 128-row block, each running the MMAs
// of all N / 256 column chunks: pass 0 takes each row's max x (and whether any x is non-finite),
// pass 1 quantises and writes the int8 row.  Rows that the certified path cannot take (a
// non-finite x, or gelu_ref(max x) below GELU_NEG_MAX, where the maximum may lie on the negative
// side) go to a list that gelu_q_rows_exact_k then computes with the exact GELU.
//
// Roles as in gemm_i8_tc: warp 0 the TMA producer (the A block is reloaded for every chunk; it
// stays in L2), warp 1 the MMA issuer (two TMEM accumulators of 256 columns), warps 2..17 the
// epilogue: warp w reads TMEM lane quarter w % 4 (thread = row) and quarter (w - 2) / 4 of each
// chunk's columns, 16 at a time.  Sixteen epilogue warps (four per scheduler) because the GELU
// and rounding work is latency-bound with fewer (measured: 8 warps left the issue slots 37 %
// busy).  The four warps of a lane quarter combine their parts of the row maxima through shared
// memory and an mbarrier (bounded wait, never a named barrier, so that a warp that gives up
// cannot leave the others waiting).
#pragma once

#include "gemm.cuh"

namespace wasr {

struct GqCfg {
  static constexpr int BM = 128, BN = 256, BK = 128;
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = 4;
  static constexpr int EPI_WARPS = 16;
  static constexpr int PARTS = EPI_WARPS / 4;  // column parts of a chunk per lane quarter
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int NMAX = 2048;  // output columns the staged column constants cover
  static constexpr int XCH = 2 * PARTS * BM * 2;  // [row-block parity][part][row][max x, check]
  static constexpr int NBAR = 2 * STAGES + 4 + 8;
  static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + (2 * NMAX + XCH) * 4 + NBAR * 8 + 16;
  static_assert(SMEM <= 232448, "shared memory");
};

// 32 lanes x 16 consecutive 32-bit TMEM columns, split into issue and wait like tmem_ld32_*.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld16_wait(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Quantised elements a rounding test could not settle: quantise them from the exact GELU.
__device__ __noinline__ void gq_requant(const float* x, float inv, uint32_t amb, uint32_t* w) {
  while (amb) {
    const int j = __ffs(amb) - 1;
    amb &= amb - 1;
    const uint32_t q = static_cast<uint8_t>(quant_one(gelu_ref(x[j]), inv));
    const int sh = 8 * (j & 3);
    w[j >> 2] = (w[j >> 2] & ~(0xffu << sh)) | (q << sh);
  }
}

// 16 consecutive outputs of one row: GELU approximation, rounding test, int8 bytes (see the
// standalone certified GELU kernel for the rounding argument), one 16-byte store.  Each element
// sets its own bit of the ambiguity mask: one running maximum of |d| over the block instead made
// the eight GELU chains of a block depend on one another and was measured 1.3x slower.
__device__ __forceinline__ void gq_quant_store(const float (&x)[16], float inv, float lim, int8_t* dst) {
  uint32_t w[4];
  uint32_t amb = 0;
  const float2 inv2 = f2c(inv), mg = f2c(RINT_MAGIC);
#pragma unroll
  for (int p4 = 0; p4 < 4; p4++) {
    uint32_t bb[4];
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int j = 4 * p4 + 2 * h;
      const float2 gg = gelu_fast2(make_float2(x[j], x[j + 1]));
      const float2 sv = fma2_rn(gg, inv2, mg);
      const float2 d = fma2_rn(gg, inv2, psub2(mg, sv));
      amb |= static_cast<uint32_t>(!(fabsf(d.x) < lim)) << j;
      amb |= static_cast<uint32_t>(!(fabsf(d.y) < lim)) << (j + 1);
      bb[2 * h] = __float_as_uint(sv.x);
      bb[2 * h + 1] = __float_as_uint(sv.y);
    }
    w[p4] = __byte_perm(__byte_perm(bb[0], bb[1], 0x0040), __byte_perm(bb[2], bb[3], 0x0040), 0x5410);
  }
  if (amb) {  // rare: the elements go through local memory to one rolled copy of the exact GELU
    float xl[16];
    uint32_t wl[4];
#pragma unroll
    for (int j = 0; j < 16; j++) xl[j] = x[j];
#pragma unroll
    for (int k = 0; k < 4; k++) wl[k] = w[k];
    gq_requant(xl, inv, amb, wl);
#pragma unroll
    for (int k = 0; k < 4; k++) w[k] = wl[k];
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(GqCfg::THREADS, 1)
    gemm_i8_gelu_q(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, GemmArgs g) {
  using Cfg = GqCfg;
  constexpr int ST = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * Cfg::A_BYTES;
  float* cws = reinterpret_cast<float*>(sB + ST * Cfg::B_BYTES);  // [NMAX] column scales
  float* cbs = cws + Cfg::NMAX;                                     // [NMAX] column biases
  float* xch = cbs + Cfg::NMAX;                                     // row maxima exchange
  uint64_t* full = reinterpret_cast<uint64_t*>(xch + Cfg::XCH);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;   // [2] accumulator ready (MMA -> epilogue)
  uint64_t* tempty = tfull + 2;   // [2] accumulator drained (epilogue -> MMA)
  uint64_t* xbar = tempty + 2;    // [row-block parity][lane quarter]: every part's maxima written
  uint32_t* tslot = reinterpret_cast<uint32_t*>(xbar + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsp = g.n_store / Cfg::BN;  // column chunks per pass
  const int steps = 2 * nsp;
  const int blocks = (g.M + Cfg::BM - 1) / Cfg::BM;
  const int nk = g.K / Cfg::BK;
  const unsigned long long lim = g.wait_ns ? g.wait_ns : WAIT_LIMIT_NS;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; s++) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, Cfg::EPI_WARPS);
    }
    for (int b = 0; b < 8; b++) mbar_init(xbar + b, Cfg::PARTS);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(tslot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  for (int c = threadIdx.x; c < g.n_store; c += blockDim.x) {
    cws[c] = g.ws_vec ? g.ws_vec[c] : g.ws;
    cbs[c] = g.bias ? g.bias[c] : 0.0f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      int kc = 0;
      for (int rb = blockIdx.x; rb < blocks && !*abort_flag && !g.idle_producer; rb += gridDim.x) {
        for (int st = 0; st < steps && !*abort_flag; st++) {
          const int n0 = (st % nsp) * Cfg::BN;
          for (int kb = 0; kb < nk; kb++, kc++) {
            const int s = kc % ST;
            if (kc >= ST && !mbar_wait(empty + s, ((kc / ST) - 1) & 1, lim)) {
              atomicExch(g.err, ERR_WAIT_EMPTY);
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(full + s, Cfg::STAGE_BYTES);
            tma_load_2d(sA + s * Cfg::A_BYTES, &tma_a, full + s, kb * Cfg::BK, rb * Cfg::BM);
            tma_load_2d(sB + s * Cfg::B_BYTES, &tma_b, full + s, kb * Cfg::BK, n0);
          }
        }
      }
      // drain: never leave the CTA while a bulk copy may still write its shared memory
      for (int k = kc > ST ? kc - ST : 0; k < kc; k++)
        if (!mbar_wait(full + k % ST, (k / ST) & 1, lim)) atomicExch(g.err, ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(Cfg::BN);
      int kc = 0, it = 0;
      for (int rb = blockIdx.x; rb < blocks && !*abort_flag; rb += gridDim.x) {
        for (int st = 0; st < steps && !*abort_flag; st++, it++) {
          const int b = it & 1, u = it >> 1;
          if (it >= 2 && !mbar_wait(tempty + b, (u - 1) & 1, lim)) {
            atomicExch(g.err, ERR_WAIT_ACC);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(b * Cfg::BN);
          for (int kb = 0; kb < nk; kb++, kc++) {
            const int s = kc % ST;
            if (!mbar_wait(full + s, (kc / ST) & 1, lim)) {
              atomicExch(g.err, ERR_WAIT_FULL);
              *abort_flag = 1;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(sA + s * Cfg::A_BYTES), b0 = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
            for (int kk = 0; kk < Cfg::BK / 32; kk++)
              mma_i8(d, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), idesc, (kb | kk) != 0);
            mma_commit(empty + s);
          }
          mma_commit(tfull + b);  // also on abort: the epilogue must not wait for nothing
        }
      }
    }
  } else {
    const int e = warp - 2, q = warp & 3, part = e >> 2;
    constexpr int PW = Cfg::BN / Cfg::PARTS;  // columns of a chunk per warp
    constexpr int SUB = PW / 16;              // 16-column loads per chunk
    static_assert(SUB % 2 == 0, "the loads alternate between two register sets");
    int it = 0, k = 0;
    bool stop = false;
    for (int rb = blockIdx.x; rb < blocks && !stop; rb += gridDim.x, k++) {
      const int row = rb * Cfg::BM + q * 32 + lane;
      const bool live = row < g.M;
      const float xs_row = live ? g.xs[row] : 0.0f;
      float xm = -3.40282347e+38f;
      float2 chk = make_float2(0.0f, 0.0f);  // stays 0 unless some x is inf or NaN
      bool fix = true;
      float inv = 1.0f, qlim = 0.0f;
      for (int st = 0; st < steps; st++, it++) {
        const int b = it & 1, u = it >> 1;
        if (st == nsp) {  // pass 0 done: the row's max over all parts -> scale and bound
          float* xk = xch + (k & 1) * (Cfg::PARTS * 2 * Cfg::BM) + 2 * (q * 32 + lane);
          xk[part * 2 * Cfg::BM] = xm;
          xk[part * 2 * Cfg::BM + 1] = __fadd_rn(chk.x, chk.y);
          __syncwarp();
          uint64_t* xb = xbar + (k & 1) * 4 + q;
          if (lane == 0) mbar_arrive(xb);
          const bool okx = mbar_wait(xb, (k >> 1) & 1, lim);
          if (!okx) {
            atomicExch(g.err, ERR_WAIT_ACC);
            *abort_flag = 1;
          }
          if (__any_sync(0xffffffffu, !okx)) {
            stop = true;
            break;
          }
          float ck = 0.0f;
#pragma unroll
          for (int p = 0; p < Cfg::PARTS; p++) {
            xm = fmaxf(xm, xk[p * 2 * Cfg::BM]);
            ck = __fadd_rn(ck, xk[p * 2 * Cfg::BM + 1]);
          }
          if (live) {
            const float mx = gelu_ref(xm);
            fix = !(ck == 0.0f) || !(mx >= GELU_NEG_MAX);
            if (!fix) {
              const float E =
                  __fmaf_ru(GELU_CERT_B, __fmul_ru(__fadd_ru(mx, GELU_CERT_A), 1.0f + 2.0f * GELU_CERT_B), GELU_CERT_A);
              const float sc = quant_scale(mx);
              inv = quant_inv(sc);
              qlim = __fsub_rd(0.5f, __fadd_ru(__fmul_ru(E, inv), 0x1p-16f));
              if (part == 0) g.q_scale[row] = sc;
            } else if (part == 0) {
              const int slot = atomicAdd(g.fix, 1);
              g.fix[1 + slot] = row;
            }
          }
        }
        const bool ok = mbar_wait(tfull + b, u & 1, lim);
        if (!ok) {
          atomicExch(g.err, ERR_WAIT_ACC);
          *abort_flag = 1;
        }
        // lanes may leave the wait apart and tcgen05.ld is .sync.aligned: decide warp-uniformly
        const bool stopw = __any_sync(0xffffffffu, !ok || *abort_flag);
        tc_fence_after();
        if (stopw) {
          stop = true;
          break;
        }
        const int n0 = (st % nsp) * Cfg::BN + part * PW;
        const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * Cfg::BN + part * PW);
        const bool pass1 = st >= nsp;
        uint32_t ra[16], rb2[16];
        tmem_ld16_issue(trow, ra);
        tmem_ld16_wait(ra);
        // one 16-column block: dequantise, then pass 0's max or pass 1's quantisation
        auto block = [&](const uint32_t(&r)[16], int col0) {
          float x[16];
#pragma unroll
          for (int j4 = 0; j4 < 4; j4++) {
            const float4 w4 = *reinterpret_cast<const float4*>(cws + col0 + 4 * j4);
            const float4 b4 = *reinterpret_cast<const float4*>(cbs + col0 + 4 * j4);
            x[4 * j4] = dequant(static_cast<int32_t>(r[4 * j4]), xs_row, w4.x, b4.x);
            x[4 * j4 + 1] = dequant(static_cast<int32_t>(r[4 * j4 + 1]), xs_row, w4.y, b4.y);
            x[4 * j4 + 2] = dequant(static_cast<int32_t>(r[4 * j4 + 2]), xs_row, w4.z, b4.z);
            x[4 * j4 + 3] = dequant(static_cast<int32_t>(r[4 * j4 + 3]), xs_row, w4.w, b4.w);
          }
          if (!pass1) {
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              xm = fmaxf(xm, fmaxf(x[j], x[j + 1]));
              chk = fma2_rn(make_float2(x[j], x[j + 1]), f2c(0.0f), chk);
            }
          } else if (live && !fix) {
            gq_quant_store(x, inv, qlim, g.q_out + static_cast<int64_t>(row) * g.n_store + col0);
          }
        };
#pragma unroll 1
        for (int c = 0; c < SUB; c += 2) {
          tmem_ld16_issue(trow + static_cast<uint32_t>(16 * (c + 1)), rb2);
          block(ra, n0 + 16 * c);
          tmem_ld16_wait(rb2);
          if (c + 2 < SUB) tmem_ld16_issue(trow + static_cast<uint32_t>(16 * (c + 2)), ra);
          block(rb2, n0 + 16 * (c + 1));
          if (c + 2 < SUB) tmem_ld16_wait(ra);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty + b);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();  // lane 0 ran the MMA loop alone: reconverge before the .sync.aligned dealloc
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

// The rows gemm_i8_gelu_q listed (g.fix[0] of them, g.fix[1..]): exact int32 dot products on the
// CUDA cores, the exact GELU and the row quantisation in the reference's order of operations.
// One block of 256 threads per listed row; the grid strides over the list (empty: no work).
__global__ void __launch_bounds__(256) gelu_q_rows_exact_k(GemmArgs g) {
  __shared__ __align__(16) int8_t arow[2048];
  __shared__ float wmax[8];
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const int cnt = g.fix[0];
  constexpr int CPT = GqCfg::NMAX / 256;
  for (int i = blockIdx.x; i < cnt; i += gridDim.x) {
    const int row = g.fix[1 + i];
    __syncthreads();  // the previous row's arow and wmax are consumed
    for (int k = tid; k < g.K; k += 256) arow[k] = g.a[static_cast<int64_t>(row) * g.K + k];
    __syncthreads();
    const float xs = g.xs[row];
    float gv[CPT];
    float mx = 0.0f;
#pragma unroll
    for (int t = 0; t < CPT; t++) {
      const int col = tid + 256 * t;
      gv[t] = 0.0f;
      if (col < g.n_store) {
        const int8_t* wr = g.b + static_cast<int64_t>(col) * g.K;
        int acc = 0;
        for (int k = 0; k < g.K; k += 4)
          acc = __dp4a(*reinterpret_cast<const int*>(arow + k), *reinterpret_cast<const int*>(wr + k), acc);
        const float ws = g.ws_vec ? g.ws_vec[col] : g.ws;
        const float bb = g.bias ? g.bias[col] : 0.0f;
        gv[t] = gelu_ref(dequant(acc, xs, ws, bb));
        mx = fmaxf(mx, fabsf(gv[t]));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) wmax[wp] = mx;
    __syncthreads();
    mx = wmax[0];
#pragma unroll
    for (int w = 1; w < 8; w++) mx = fmaxf(mx, wmax[w]);
    const float sc = quant_scale(mx), inv = quant_inv(sc);
#pragma unroll
    for (int t = 0; t < CPT; t++) {
      const int col = tid + 256 * t;
      if (col < g.n_store) g.q_out[static_cast<int64_t>(row) * g.n_store + col] = quant_one(gv[t], inv);
    }
    if (tid == 0) g.q_scale[row] = sc;
  }
}

}  // namespace wasr
