// gemm.cuh -- int8 x int8 -> int32 GEMM on the 5th-generation tensor cores (tcgen05,
// kind::i8) with fused epilogues, replacing the reference's cuBLASLt call plus its separate
// epilogue kernels (csrc/wtlgpu.cu:249-380,533-626).
//
//   acc[i][j] = sum_k A[i][k] * B[j][k]        A = activations [M][K], B = weights [N][K]
//
// Both operands are K-major (row-major [rows][K]), exactly the layout of the reference's
// xq buffers and blob weights, so TMA loads them directly with 128-byte swizzle into the
// canonical UMMA K-major layout.  CTAs are persistent over 128 x BN tiles:
//   warp 0      : TMA producer (one elected lane), STAGES-deep smem ring
//   warp 1      : TMEM allocator + MMA issuer (one lane issues tcgen05.mma, M=128, N=BN, K=32)
//   warps 2..9  : epilogue; warp w reads TMEM lanes 32*(w%4).. with tcgen05.ld (thread = row),
//                 writes each 32 x 32 block into a 128-byte-swizzled staging buffer and TMA-stores
//                 it (residual epilogue: the h block arrives by TMA load two blocks ahead)
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
  EPI_GELU_Q = 6,      // int8 rows + scales of quant(gelu(out)), out never stored (gemm_gq.cuh)
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
  int tma_out;         // 1: out / out_i32 blocks move by TMA (tensor map passed to the kernel)
  unsigned long long wait_ns;  // limit of every mbarrier wait (0: WAIT_LIMIT_NS)
  int idle_producer;   // failure-handling test only: the producer issues no loads, so the
                       // consumers' waits run out with nothing in flight
  int8_t* q_out;       // EPI_GELU_Q: int8 rows [M][n_store]
  float* q_scale;      // EPI_GELU_Q: row scales [M]
  int* fix;            // EPI_GELU_Q: [1 + M] ints, the count and the rows left to the exact kernel
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

// EW: epilogue warps, 8 (two per TMEM lane quarter, half the columns each) or 4 (one per
// quarter, all columns) -- the latter frees shared memory for deeper K pipelines.
template <int BN, int EPI, int EW = 8>
struct TcCfg {
  static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
  static constexpr int BM = 128;
  static constexpr int BK = 128;  // bytes of K per stage = one 128-byte swizzle row
  static constexpr int A_BYTES = BM * BK;
  static constexpr int B_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // staging buffers per epilogue warp: 2 for stores, 3 when h blocks are loaded ahead as well
  static constexpr int NBUF = EPI == EPI_F32_ADD ? 3 : 2;
  static constexpr int STAGES = EW == 4 ? 5 : BN >= 256 ? (EPI == EPI_F32_ADD ? 2 : 3) : (EPI == EPI_F32_ADD && BN == 128 ? 3 : 4);
  static_assert(EW == 8 || EW == 4, "epilogue warps");
  static constexpr int EPI_WARPS = EW;
  static constexpr int HALVES = EW / 4;               // column halves of a tile per lane quarter
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int TMEM_COLS = 2 * BN;            // two accumulator buffers
  static constexpr int STG_FLOATS = 32 * 32;          // one 32 x 32 block (4 KB, 1024-byte aligned)
  static constexpr int COLC = 64;                     // per epilogue warp: 32 column scales + 32 biases
  static constexpr int NBAR = 2 * STAGES + 4 + EPI_WARPS * NBUF;
  static constexpr int SMEM =
      1024 + STAGES * STAGE_BYTES + EPI_WARPS * (NBUF * STG_FLOATS + COLC) * 4 + NBAR * 8 + 16;
  static_assert(SMEM <= 232448, "shared memory");
};

// Epilogue staging: a warp's 32 rows x 32 columns, stored so that row-per-thread float4
// writes and row-contiguous float4 reads (8 lanes per 128-byte row segment) are both at the
// minimum number of shared-memory wavefronts (16-byte groups XOR-swizzled by row).
__device__ __forceinline__ int stg_off(int r, int c4) { return r * 32 + ((c4 ^ (r & 7)) << 2); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One 32-column chunk of a warp's 32 rows.  r[] holds row (rowbase + lane), columns
// col0..col0+31 of the accumulator; columns >= n_store and rows >= M are never written.
template <int EPI>
__device__ __forceinline__ void epi_chunk(const GemmArgs& g, float* stg, int lane, int rowbase, int col0,
                                          const uint32_t (&r)[32], float& rmax, float& best, uint32_t& bidx) {
  const int row = rowbase + lane;
  const int ncols = min(32, g.n_store - col0);
  if constexpr (EPI == EPI_ARGMAX) {
    if (row < g.M) {
      const float xs = g.xs[row];
#pragma unroll
      for (int j = 0; j < 32; j++) {
        if (j < ncols) {
          const int col = col0 + j;
          const float ws = g.ws_vec ? __ldg(g.ws_vec + col) : g.ws;
          const float bb = g.bias ? __ldg(g.bias + col) : 0.0f;
          const float v = dequant(static_cast<int32_t>(r[j]), xs, ws, bb);
          if (v > best) { best = v; bidx = static_cast<uint32_t>(col); }
        }
      }
    }
    return;
  } else {
    float v[32];
    if constexpr (EPI == EPI_I32) {
#pragma unroll
      for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
    } else {
      const float xs = row < g.M ? g.xs[row] : 0.0f;
#pragma unroll
      for (int j = 0; j < 32; j++) {
        const int col = col0 + j;
        const bool in = j < ncols;
        const float ws = !in ? 0.0f : g.ws_vec ? __ldg(g.ws_vec + col) : g.ws;
        const float bb = (in && g.bias) ? __ldg(g.bias + col) : 0.0f;
        v[j] = dequant(static_cast<int32_t>(r[j]), xs, ws, bb);
        if constexpr (EPI == EPI_F32_ROWMAX) {
          if (in) rmax = fmaxf(rmax, fabsf(v[j]));
        }
      }
    }
#pragma unroll
    for (int c4 = 0; c4 < 8; c4++)
      *reinterpret_cast<float4*>(stg + stg_off(lane, c4)) = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
    if constexpr (EPI == EPI_GELU_ROWMAX) {
      // GELU in place, rolled (the exact tanh is long: one copy of its code, not 32)
#pragma unroll 1
      for (int j = 0; j < 32; j++) {
        const int off = stg_off(lane, j >> 2) + (j & 3);
        const float gv = gelu_ref(stg[off]);
        stg[off] = gv;
        if (j < ncols) rmax = fmaxf(rmax, fabsf(gv));
      }
    }
    __syncwarp();
    // coalesced write-out: lane -> (row group lane/8, 4-column group lane%8), 4 rows per pass
    const int c4 = lane & 7;
    const int col = col0 + 4 * c4;
    const bool vec = (g.ldo & 3) == 0 && col + 3 < g.n_store;
#pragma unroll 2
    for (int i = 0; i < 8; i++) {
      const int rr = 4 * i + (lane >> 3);
      const int grow = rowbase + rr;
      if (grow < g.M && col < g.n_store) {
        const float4 x = *reinterpret_cast<const float4*>(stg + stg_off(rr, c4));
        const int64_t o = static_cast<int64_t>(grow) * g.ldo + col;
        if constexpr (EPI == EPI_I32) {
          if (vec) {
            *reinterpret_cast<int4*>(g.out_i32 + o) =
                make_int4(__float_as_int(x.x), __float_as_int(x.y), __float_as_int(x.z), __float_as_int(x.w));
          } else {
            const float xv[4] = {x.x, x.y, x.z, x.w};
            for (int k = 0; k < 4 && col + k < g.n_store; k++) g.out_i32[o + k] = __float_as_int(xv[k]);
          }
        } else if constexpr (EPI == EPI_F32_ADD) {
          if (vec) {
            const float4 h = *reinterpret_cast<const float4*>(g.out + o);
            *reinterpret_cast<float4*>(g.out + o) =
                make_float4(__fadd_rn(h.x, x.x), __fadd_rn(h.y, x.y), __fadd_rn(h.z, x.z), __fadd_rn(h.w, x.w));
          } else {
            const float xv[4] = {x.x, x.y, x.z, x.w};
            for (int k = 0; k < 4 && col + k < g.n_store; k++) g.out[o + k] = __fadd_rn(g.out[o + k], xv[k]);
          }
        } else {
          if (vec) {
            *reinterpret_cast<float4*>(g.out + o) = x;
          } else {
            const float xv[4] = {x.x, x.y, x.z, x.w};
            for (int k = 0; k < 4 && col + k < g.n_store; k++) g.out[o + k] = xv[k];
          }
        }
      }
    }
    __syncwarp();  // the staging buffer is reused by the next chunk
  }
}

// The argmax epilogue of one 32-column chunk of this thread's row (output layer, src/model.rs:
// 498-501): v = (acc * xs) * ws[col] + bias[col], then the first maximum.  The chunk's column
// scales / biases come from the warp's staged colc (four at a time, the same address for every
// lane); two interleaved partial maxima (4-column groups alternately) shorten the dependent
// compare chain and merge with first-max-wins; columns >= n_store (the tail chunk) never win.
__device__ __forceinline__ void argmax_upd(float v, uint32_t c, float& b, uint32_t& i) {
  const bool w = v > b;
  b = w ? v : b;
  i = w ? c : i;
}
template <bool FULL>
__device__ __forceinline__ void epi_argmax_chunk(const GemmArgs& g, const float* colc, bool cw, bool cb, float xs,
                                                 int col0, const uint32_t (&r)[32], float& best, uint32_t& bidx) {
  const int ncols = FULL ? 32 : min(32, g.n_store - col0);
  float b2 = -3.40282347e+38f;
  uint32_t i2 = 0xFFFFFFFFu;
#pragma unroll
  for (int j4 = 0; j4 < 8; j4++) {
    const float4 w4 = cw ? *reinterpret_cast<const float4*>(colc + 4 * j4) : make_float4(g.ws, g.ws, g.ws, g.ws);
    const float4 c4 = cb ? *reinterpret_cast<const float4*>(colc + 32 + 4 * j4) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float wk[4] = {w4.x, w4.y, w4.z, w4.w}, bk[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int j = 4 * j4 + k;
      float v = dequant(static_cast<int32_t>(r[j]), xs, wk[k], bk[k]);
      if (!FULL) v = j < ncols ? v : -__int_as_float(0x7f800000);  // never beats -FLT_MAX
      if (j4 & 1) argmax_upd(v, static_cast<uint32_t>(col0 + j), b2, i2);
      else argmax_upd(v, static_cast<uint32_t>(col0 + j), best, bidx);
    }
  }
  // merge: the larger value wins; equal values keep the lower column
  const bool take = b2 > best || (b2 == best && i2 < bidx);
  best = take ? b2 : best;
  bidx = take ? i2 : bidx;
}

// One 32 x 32 block on the TMA path: thread `lane` owns row `row` (columns col0..col0+31).
// On entry `buf` holds the block's h values (EPI_F32_ADD); on exit it holds the output block
// in the 128-byte-swizzled layout of the output tensor map.  Columns >= n_store and rows
// >= M are computed from zero scales and clipped by the store.
template <int EPI>
__device__ __forceinline__ void epi_block_tma(const GemmArgs& g, float* buf, const float* colc, float xs, int lane,
                                              int col0, const uint32_t (&r)[32], float& rmax) {
  // colc[0..31] / colc[32..63]: per-channel scale / bias of columns col0.. (0 past n_store)
  const int ncols = min(32, g.n_store - col0);
  float v[32];
  if constexpr (EPI == EPI_I32) {
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
  } else {
    const bool has_wv = g.ws_vec != nullptr, has_b = g.bias != nullptr;
#pragma unroll
    for (int j4 = 0; j4 < 8; j4++) {
      const float4 w4 = has_wv ? *reinterpret_cast<const float4*>(colc + 4 * j4) : make_float4(g.ws, g.ws, g.ws, g.ws);
      const float4 b4 = has_b ? *reinterpret_cast<const float4*>(colc + 32 + 4 * j4) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float wk[4] = {w4.x, w4.y, w4.z, w4.w}, bk[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int j = 4 * j4 + k;
        // columns past n_store have zero accumulators (the weight rows past N are zero-filled
        // by TMA) and zero staged constants; the store clips them, only the row max skips them
        v[j] = dequant(static_cast<int32_t>(r[j]), xs, wk[k], bk[k]);
        if constexpr (EPI == EPI_F32_ROWMAX) {
          if (j < ncols) rmax = fmaxf(rmax, fabsf(v[j]));
        }
      }
    }
  }
#pragma unroll
  for (int c4 = 0; c4 < 8; c4++) {
    float4* p = reinterpret_cast<float4*>(buf + stg_off(lane, c4));
    float4 w = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
    if constexpr (EPI == EPI_F32_ADD) {
      const float4 h = *p;  // h + o, src/model.rs:493,496
      w = make_float4(__fadd_rn(h.x, w.x), __fadd_rn(h.y, w.y), __fadd_rn(h.z, w.z), __fadd_rn(h.w, w.w));
    }
    *p = w;
  }
  if constexpr (EPI == EPI_GELU_ROWMAX) {
    // 8 columns per step as 4 packed pairs: the exact tanh chains (hundreds of cycles each)
    // overlap instead of running one after another
#pragma unroll 1
    for (int c4 = 0; c4 < 8; c4 += 2) {
      float4* p0 = reinterpret_cast<float4*>(buf + stg_off(lane, c4));
      float4* p1 = reinterpret_cast<float4*>(buf + stg_off(lane, c4 + 1));
      const float4 a = *p0, b = *p1;
      const float2 g0 = gelu_ref2(make_float2(a.x, a.y)), g1 = gelu_ref2(make_float2(a.z, a.w));
      const float2 g2 = gelu_ref2(make_float2(b.x, b.y)), g3 = gelu_ref2(make_float2(b.z, b.w));
      *p0 = make_float4(g0.x, g0.y, g1.x, g1.y);
      *p1 = make_float4(g2.x, g2.y, g3.x, g3.y);
      const float gv[8] = {g0.x, g0.y, g1.x, g1.y, g2.x, g2.y, g3.x, g3.y};
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (4 * c4 + u < ncols) rmax = fmaxf(rmax, fabsf(gv[u]));
    }
  }
}

// Persistent, warp-specialised tcgen05 GEMM.  CTAs walk the 128 x BN output tiles in a
// static round robin.  Warp 0 (one lane) streams A/B k-blocks through a STAGES-deep TMA ring;
// warp 1 (one lane) issues tcgen05.mma into one of two TMEM accumulators; warps 2..9 drain the
// other accumulator, so a tile's epilogue overlaps the next tile's MMAs.  Each epilogue warp
// walks its sequence of 32 x 32 output blocks (BN/64 per tile); on the TMA path block cc is
// staged in buffer cc % NBUF and stored with one bulk tensor store, and for the residual
// epilogue lane 0 loads the h block of cc+2 as soon as its buffer's last store has read it.
template <int BN, int EPI, int EW = 8>
__global__ void __launch_bounds__(TcCfg<BN, EPI, EW>::THREADS, 1)
    gemm_i8_tc(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
               const __grid_constant__ CUtensorMap tma_o, GemmArgs g) {
  using Cfg = TcCfg<BN, EPI, EW>;
  constexpr int ST = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + ST * Cfg::A_BYTES;
  float* stg_all = reinterpret_cast<float*>(sB + ST * Cfg::B_BYTES);
  float* colc_all = stg_all + Cfg::EPI_WARPS * Cfg::NBUF * Cfg::STG_FLOATS;  // [EPI_WARPS][64]
  uint64_t* full = reinterpret_cast<uint64_t*>(colc_all + Cfg::EPI_WARPS * Cfg::COLC);
  uint64_t* empty = full + ST;
  uint64_t* tfull = empty + ST;   // [2] accumulator ready (MMA -> epilogue)
  uint64_t* tempty = tfull + 2;   // [2] accumulator drained (epilogue -> MMA)
  uint64_t* hbar = tempty + 2;    // [EPI_WARPS][NBUF] h block landed (TMA -> epilogue warp)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(hbar + Cfg::EPI_WARPS * Cfg::NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tslot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (g.n_store + BN - 1) / BN;
  const int tiles = n_tiles * ((g.M + Cfg::BM - 1) / Cfg::BM);
  // tile -> (m, n) without a run-time division: q = (tile * ceil(2^40 / n_tiles)) >> 40 is exact
  // for tile < 2^24 and n_tiles < 2^16 (the error tile / 2^40 stays below 1 / n_tiles)
  const unsigned long long tmagic = ((1ull << 40) + static_cast<unsigned>(n_tiles) - 1) / static_cast<unsigned>(n_tiles);
  auto tile_m = [&](int tile) { return static_cast<int>((static_cast<unsigned long long>(tile) * tmagic) >> 40); };
  const int nk = (g.K + Cfg::BK - 1) / Cfg::BK;
  const bool tma_out = g.tma_out != 0 && EPI != EPI_ARGMAX;
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
    for (int b = 0; b < Cfg::EPI_WARPS * Cfg::NBUF; b++) mbar_init(hbar + b, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
    if (tma_out) tma_prefetch_desc(&tma_o);
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
      int kc = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort_flag && !g.idle_producer; tile += gridDim.x) {
        const int tm = tile_m(tile);
        const int m0 = tm * Cfg::BM, n0 = (tile - tm * n_tiles) * BN;
        for (int kb = 0; kb < nk; kb++, kc++) {
          const int s = kc % ST;
          if (kc >= ST && !mbar_wait(empty + s, ((kc / ST) - 1) & 1, lim)) {
            atomicExch(g.err, ERR_WAIT_EMPTY);
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(full + s, Cfg::STAGE_BYTES);
          tma_load_2d(sA + s * Cfg::A_BYTES, &tma_a, full + s, kb * Cfg::BK, m0);
          tma_load_2d(sB + s * Cfg::B_BYTES, &tma_b, full + s, kb * Cfg::BK, n0);
        }
      }
      // drain: never leave the CTA while a bulk copy may still write its shared memory
      for (int k = kc > ST ? kc - ST : 0; k < kc; k++)
        if (!mbar_wait(full + k % ST, (k / ST) & 1, lim)) atomicExch(g.err, ERR_WAIT_FULL);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8(BN);
      int kc = 0, it = 0;
      for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x, it++) {
        const int b = it & 1, u = it >> 1;
        if (it >= 2 && !mbar_wait(tempty + b, (u - 1) & 1, lim)) {
          atomicExch(g.err, ERR_WAIT_ACC);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * BN);
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
  } else {
    const int e = warp - 2, q = warp & 3, half = e >> 2;  // TMEM lane quarter = warp % 4
    constexpr int HW = BN / Cfg::HALVES;                    // columns of a tile per warp
    float* wb = stg_all + e * Cfg::NBUF * Cfg::STG_FLOATS;
    float* colc = colc_all + e * Cfg::COLC;
    uint64_t* hb = hbar + e * Cfg::NBUF;
    constexpr int CPT = HW / 32;  // 32-column blocks per tile for this warp
    // block cc of this warp's sequence -> (first row, first column); false past the last tile
    // or past n_store
    auto block_at = [&](int cc, int& row, int& col) {
      const int k = cc / CPT;
      const int tile = blockIdx.x + k * gridDim.x;
      if (tile >= tiles) return false;
      const int tm = tile_m(tile);
      row = tm * Cfg::BM + q * 32;
      col = (tile - tm * n_tiles) * BN + half * HW + 32 * (cc - k * CPT);
      return col < g.n_store;
    };
    uint32_t hpar = 0, pend = 0;  // per-buffer phase parity (all lanes); loads in flight (lane 0)
    auto load_h = [&](int cc) {   // lane 0 only
      int row, col;
      if (!block_at(cc, row, col)) return;
      const int bi = cc % Cfg::NBUF;
      mbar_arrive_expect_tx(hb + bi, Cfg::STG_FLOATS * 4);
      tma_load_2d(wb + bi * Cfg::STG_FLOATS, &tma_o, hb + bi, col, row);
      pend |= 1u << bi;
    };
    // with the long-K configuration (4 epilogue warps), h blocks one tile ahead of their load
    // are prefetched into L2 (measured: a gain there, a loss with 8 warps and K = 512)
    auto prefetch_h = [&](int cc) {  // lane 0 only
      int row, col;
      if (EW == 4 && block_at(cc, row, col)) tma_prefetch_2d(&tma_o, col, row);
    };
    if constexpr (EPI == EPI_F32_ADD) {
      if (tma_out && lane == 0) {
        load_h(0);
        load_h(1);
        for (int j = 2; j < 2 + CPT; j++) prefetch_h(j);
      }
    }
    // column constants (per-channel scale, bias) of the next block, one per lane, fetched a
    // block ahead so the loads never stall the dequant
    const bool colconst = (tma_out || EPI == EPI_ARGMAX) && EPI != EPI_I32 && (g.ws_vec || g.bias);
    float nws = 0.0f, nbias = 0.0f;
    auto fetch_cols = [&](int cc) {
      int row, col;
      nws = nbias = 0.0f;
      if (!block_at(cc, row, col) || col + lane >= g.n_store) return;
      if (g.ws_vec) nws = __ldg(g.ws_vec + col + lane);
      if (g.bias) nbias = __ldg(g.bias + col + lane);
    };
    if (colconst) fetch_cols(0);
    int it = 0, cc = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, it++) {
      const int b = it & 1, u = it >> 1;
      const int tm = tile_m(tile);
      const int m0 = tm * Cfg::BM, n0 = (tile - tm * n_tiles) * BN;
      // this thread's row scale, loaded while the accumulator is still being computed
      const float xs_row = (EPI != EPI_I32 && m0 + q * 32 + lane < g.M) ? g.xs[m0 + q * 32 + lane] : 0.0f;
      const bool ok = mbar_wait(tfull + b, u & 1, lim);
      if (!ok) {
        atomicExch(g.err, ERR_WAIT_ACC);
        *abort_flag = 1;
      }
      // lanes may leave the wait apart and tcgen05.ld is .sync.aligned: decide warp-uniformly
      const bool stop = __any_sync(0xffffffffu, !ok || *abort_flag);
      tc_fence_after();
      if (stop) break;
      const int rowbase = m0 + q * 32;
      float rmax = 0.0f, best = -3.40282347e+38f;
      uint32_t bidx = 0xFFFFFFFFu;
      // the accumulator chunk c + 1 is read from TMEM while chunk c is processed (measured: a gain
      // for the fp32 and 8-warp residual epilogues, a loss for the 4-warp one and the argmax)
      constexpr bool kOverlap = EPI == EPI_F32 || (EPI == EPI_F32_ADD && EW == 8);
      const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BN + half * HW);
      uint32_t ra[32], rb[32];
      tmem_ld32_issue(trow, ra);
      tmem_ld32_wait(ra);
#pragma unroll(kOverlap ? CPT : 1)
      for (int c = 0; c < CPT; c++, cc++) {
        const int c0 = half * HW + 32 * c;
        const int col = n0 + c0;
        uint32_t(&r)[32] = (kOverlap && (c & 1)) ? rb : ra;
        uint32_t(&rn)[32] = (kOverlap && (c & 1)) ? ra : rb;
        if (kOverlap && c + 1 < CPT) tmem_ld32_issue(trow + static_cast<uint32_t>(32 * (c + 1)), rn);
        if (!kOverlap && c > 0) {
          tmem_ld32_issue(trow + static_cast<uint32_t>(32 * c), r);
          tmem_ld32_wait(r);
        }
        if (colconst) {
          colc[lane] = nws;
          colc[32 + lane] = nbias;
          __syncwarp();
          fetch_cols(cc + 1);
        }
        if (col < g.n_store) {
          if (tma_out) {
            const int bi = cc % Cfg::NBUF;
            float* buf = wb + bi * Cfg::STG_FLOATS;
            if constexpr (EPI == EPI_F32_ADD) {
              if (!mbar_wait(hb + bi, (hpar >> bi) & 1, lim)) {
                atomicExch(g.err, ERR_WAIT_FULL);
                *abort_flag = 1;
              }
              hpar ^= 1u << bi;
              if (lane == 0) pend &= ~(1u << bi);
            } else {
              if (lane == 0) bulk_wait_read<Cfg::NBUF - 1>();  // the store of block cc-NBUF has read buf
              __syncwarp();
            }
            epi_block_tma<EPI>(g, buf, colc, xs_row, lane, col, r, rmax);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tma_o, buf, col, rowbase);
              bulk_commit();
            }
          } else {
            if constexpr (EPI == EPI_ARGMAX) {
              if (rowbase + lane < g.M) {
                if (col + 32 <= g.n_store)
                  epi_argmax_chunk<true>(g, colc, g.ws_vec != nullptr, g.bias != nullptr, xs_row, col, r, best, bidx);
                else
                  epi_argmax_chunk<false>(g, colc, g.ws_vec != nullptr, g.bias != nullptr, xs_row, col, r, best, bidx);
              }
              __syncwarp();  // colc is rewritten for the next chunk
            } else {
              epi_chunk<EPI>(g, wb, lane, rowbase, col, r, rmax, best, bidx);
            }
          }
        }
        if constexpr (EPI == EPI_F32_ADD) {
          if (tma_out && lane == 0) {
            bulk_wait_read<1>();  // buffer (cc+2) % 3 was last read by the store of block cc-1
            load_h(cc + 2);
            prefetch_h(cc + 2 + CPT);
          }
        }
        if (kOverlap && c + 1 < CPT) tmem_ld32_wait(rn);
      }
      if (rowbase + lane < g.M) epi_finish_row<EPI>(g, rowbase + lane, rmax, best, bidx);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + b);
    }
    if (tma_out && lane == 0) {
      bulk_wait_all();
      // h loads issued ahead but never consumed (abort): let them land before the CTA exits
      for (int bi = 0; bi < Cfg::NBUF; bi++)
        if ((pend >> bi) & 1u) mbar_wait(hb + bi, (hpar >> bi) & 1, lim);
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
// Whether gemm_run takes this EPI_GELU_Q call (K a multiple of 128 up to 2048, N a multiple of
// 256 up to 2048, 16-byte aligned operands and output, the output buffers given).
bool gemm_gq_supported(const GemmArgs& g);
// Set every kernel's shared-memory attribute on the current device (call outside capture).
bool gemm_prepare();

}  // namespace wasr
