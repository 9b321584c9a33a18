// kern.cu -- conv frontend, LayerNorm/quant/GELU/argmax and attention kernels, plus the
// reference's wk_* C ABI on top of them (csrc/wtl_kern.cu:409-462, csrc/wk_attention_*.cu).
//
// Bit-exactness: the conv frontend, LayerNorm and quantisation reproduce the CPU path's
// operation order (src/kernels.rs dotf / quant, src/model.rs norm / frontend) with
// explicitly rounded intrinsics, so their outputs equal the CPU's bit for bit.  Attention
// keeps the CPU's order too (8-lane dot, sequential softmax sum, sequential PV sum), and the
// softmax exp and the GELU tanh are restatements of glibc's algorithms (common.cuh), so they
// are bit-exact as well.
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <set>
#include <utility>

#include "../../include/wtlgpu.h"
#include "kern.cuh"

namespace wasr {

// ------------------------------------------------------------------------ conv1
// y1[g][o][f] = relu(dotf(c1[o], patch5x5(x, g, f))) -- src/model.rs:398-418.
// dotf over 25 taps: lanes 0..7 take taps l, 8+l, 16+l in order; tail = tap 24.
__global__ void __launch_bounds__(128) conv1_k(const float* __restrict__ x, const float* __restrict__ c1, Segs s,
                                               int total, float* __restrict__ y1) {
  __shared__ float w[C1 * 25];
  for (int i = threadIdx.x; i < C1 * 25; i += blockDim.x) w[i] = c1[i];
  __syncthreads();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total * DIM) return;
  const int g = idx / DIM, f = idx - g * DIM;
  const int sw = s.seg_of_frame(g);
  const int fb = s.frame_begin(sw), t = s.frames(sw), ti = g - fb;
  float p[25];
#pragma unroll
  for (int i = 0; i < 5; i++) {
    const int tt = ti + i - 2;
#pragma unroll
    for (int j = 0; j < 5; j++) {
      const int ff = f + j - 2;
      p[i * 5 + j] = (tt >= 0 && tt < t && ff >= 0 && ff < DIM) ? x[static_cast<int64_t>(fb + tt) * DIM + ff] : 0.0f;
    }
  }
  float* out = y1 + static_cast<int64_t>(g) * (C1 * DIM) + f;
#pragma unroll 4
  for (int o = 0; o < C1; o++) {
    const float* wo = w + o * 25;
    float a[8];
#pragma unroll
    for (int l = 0; l < 8; l++) a[l] = __fadd_rn(0.0f, __fmul_rn(wo[l], p[l]));
#pragma unroll
    for (int c = 1; c < 3; c++)
#pragma unroll
      for (int l = 0; l < 8; l++) a[l] = __fadd_rn(a[l], __fmul_rn(wo[c * 8 + l], p[c * 8 + l]));
    float sum = a[0];
#pragma unroll
    for (int l = 1; l < 8; l++) sum = __fadd_rn(sum, a[l]);
    const float v = __fadd_rn(sum, __fmul_rn(wo[24], p[24]));
    out[o * DIM] = fmaxf(v, 0.0f);
  }
}

// conv1 of the engine: the weights arrive as a kernel argument (a __grid_constant__ struct in the
// constant bank) and the channel loop is fully unrolled, so every multiply names its weight
// directly instead of loading it from shared memory (one load per multiply in conv1_k).
__global__ void __launch_bounds__(128) conv1w_k(const float* __restrict__ x, const __grid_constant__ Conv1W cw,
                                                Segs s, int total, float* __restrict__ y1) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= total * DIM) return;
  const int g = idx / DIM, f = idx - g * DIM;
  const int sw = s.seg_of_frame(g);
  const int fb = s.frame_begin(sw), t = s.frames(sw), ti = g - fb;
  float p[25];
#pragma unroll
  for (int i = 0; i < 5; i++) {
    const int tt = ti + i - 2;
#pragma unroll
    for (int j = 0; j < 5; j++) {
      const int ff = f + j - 2;
      p[i * 5 + j] = (tt >= 0 && tt < t && ff >= 0 && ff < DIM) ? x[static_cast<int64_t>(fb + tt) * DIM + ff] : 0.0f;
    }
  }
  float* out = y1 + static_cast<int64_t>(g) * (C1 * DIM) + f;
#pragma unroll
  for (int o = 0; o < C1; o++) {
    const float* wo = cw.w + o * 25;
    float a[8];
#pragma unroll
    for (int l = 0; l < 8; l++) a[l] = __fadd_rn(0.0f, __fmul_rn(wo[l], p[l]));
#pragma unroll
    for (int c = 1; c < 3; c++)
#pragma unroll
      for (int l = 0; l < 8; l++) a[l] = __fadd_rn(a[l], __fmul_rn(wo[c * 8 + l], p[c * 8 + l]));
    float sum = a[0];
#pragma unroll
    for (int l = 1; l < 8; l++) sum = __fadd_rn(sum, a[l]);
    const float v = __fadd_rn(sum, __fmul_rn(wo[24], p[24]));
    out[o * DIM] = fmaxf(v, 0.0f);
  }
}

// ------------------------------------------------------------------------ conv2 / conv3
// Both are dotf products of a weight row with a zero-padded patch (src/kernels.rs dotf: 8
// lane accumulators, lane l takes taps l, l+8, l+16, ... in order, then the lanes are folded
// l0 + l1 + ... + l7).  For conv2 and conv3 the patch length (1568, 576) is a multiple of 8,
// and the lane of tap idx = c*49 + i*7 + j (conv2) or c*9 + i*3 + j (conv3) is (c + rest) % 8
// because 49 = 9 = 1 mod 8.
//
// Lane-pair layout.  Taps 2m and 2m+1 land in lanes (2q, 2q+1) for one q in 0..3, so the
// 256 threads of a block form 4 groups, group q accumulating lanes 2q and 2q+1 of every
// output it owns as one float2.  For a tap pair the two weights are adjacent in memory and
// the two inputs are staged interleaved (X2[m][f] = (patch[2m](f), patch[2m+1](f))), so a
// product pair is one packed multiply of two register pairs and the accumulate one packed
// add -- every element still rounds exactly like the scalar sequence.  A thread owns
// 5 positions x 4 output channels (40 accumulator registers).  After the last stage the
// partial lanes go through shared memory and are folded in lane order.
constexpr int TP_THREADS = 256;
constexpr int TP_P = 5, TP_C = 4;  // positions x channels per thread

// Staging of a stage: every copy is issued at once with cp.async (weight pairs straight from
// the [out][tap] layout, 8 bytes each; the stage's raw input rows), waited for once, and the
// interleaved X2 is then built from shared memory through a per-block table of tap offsets.
constexpr int CV2_CH = 32;                 // output channels per block
constexpr int CV2_CC = 4;                  // input channels per stage
constexpr int CV2_MP = CV2_CC * 49 / 2;    // tap pairs per stage (98)
constexpr int CV2_WS = CV2_CH + 2;         // W2 row stride in float2 (16-byte rows)
constexpr int CV2_RW = 48;                 // raw row: 4 zeros | 40 values | 4 zeros (16-byte aligned data)
constexpr int CV2_RAW = 7 * CV2_CC * CV2_RW;
constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int CV2_PS = DIM + 2;            // partial-lane row stride in float2 (conflict-free stores)
constexpr int CV2_SMEM = cmax(CV2_MP * (DIM + CV2_WS) * 8 + CV2_RAW * 4 + 2 * CV2_MP * 4, 4 * CV2_CH * CV2_PS * 8);

constexpr int CV3_CH = 64;
constexpr int CV3_CC = 16;
constexpr int CV3_MP = CV3_CC * 9 / 2;     // 72
constexpr int CV3_WS = CV3_CH + 2;
constexpr int CV3_RW = W2;                 // raw row: the 41 values of a channel, so the 16 channels
                                           // of an input row are one contiguous 16-byte-aligned span
constexpr int CV3_RAW = 3 * CV3_CC * CV3_RW;
constexpr int CV3_PS = 21;                 // partial-lane row stride in float2 (conflict-free stores)
constexpr int CV3_SMEM = cmax(CV3_MP * (20 + CV3_WS) * 8 + CV3_RAW * 4 + 2 * CV3_MP * 4, 4 * CV3_CH * CV3_PS * 8);

__device__ __forceinline__ float2 mulp(float2 a, float2 b) {
  return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
}

// acc[p][c] += X2[m][f0+p] * W2[m][o0+c] for this group's tap pairs m = m0, m0+4, ... < mp
template <int XS, int WS, int UNROLL>
__device__ __forceinline__ void tp_accumulate(const float2* __restrict__ X2, const float2* __restrict__ W2, int mp,
                                              int m0, int f0, int o0, float2 (&acc)[TP_P][TP_C]) {
#pragma unroll UNROLL
  for (int m = m0; m < mp; m += 4) {
    const float2* xr = X2 + m * XS + f0;
    const float4* wr = reinterpret_cast<const float4*>(W2 + m * WS + o0);
    float2 xv[TP_P];
#pragma unroll
    for (int p = 0; p < TP_P; p++) xv[p] = xr[p];
    const float4 wa = wr[0], wb = wr[1];
    const float2 wv[TP_C] = {make_float2(wa.x, wa.y), make_float2(wa.z, wa.w), make_float2(wb.x, wb.y),
                             make_float2(wb.z, wb.w)};
#pragma unroll
    for (int p = 0; p < TP_P; p++)
#pragma unroll
      for (int c = 0; c < TP_C; c++) acc[p][c] = add2_rn(acc[p][c], mulp(xv[p], wv[c]));
  }
}

// Fold the 4 groups' lane pairs of output (o, f) in lane order; part = [4][nch][npos].
__device__ __forceinline__ float tp_fold(const float2* part, int nch, int npos, int o, int f) {
  const float2 a0 = part[(0 * nch + o) * npos + f], a1 = part[(1 * nch + o) * npos + f];
  const float2 a2 = part[(2 * nch + o) * npos + f], a3 = part[(3 * nch + o) * npos + f];
  float s = __fadd_rn(a0.x, a0.y);
  s = __fadd_rn(s, a1.x);
  s = __fadd_rn(s, a1.y);
  s = __fadd_rn(s, a2.x);
  s = __fadd_rn(s, a2.y);
  s = __fadd_rn(s, a3.x);
  return __fadd_rn(s, a3.y);
}

// y2[r][o][f] = relu(dotf(c2[o], patch)), patch[c*49+i*7+j] = y1[5r+i-1][c][f+j-3] (zero
// outside the segment / the 40 columns), column 40 = 0 -- src/model.rs:420-444.
// Block = (row r, 32 output channels); stages of 4 input channels.
__global__ void __launch_bounds__(TP_THREADS, 3) conv2_k(const float* __restrict__ y1, const float* __restrict__ c2,
                                                      Segs s, int row0, float* __restrict__ y2) {
  extern __shared__ __align__(16) float sm[];
  float2* X2 = reinterpret_cast<float2*>(sm);    // [98][40]
  float2* Wt = X2 + CV2_MP * DIM;                 // [98][34]
  float* raw = reinterpret_cast<float*>(Wt + CV2_MP * CV2_WS);  // [7 rows][4 channels][48]
  int* tapoff = reinterpret_cast<int*>(raw + CV2_RAW);          // [196] tap -> raw offset (+ f)
  // the channel groups of a row are adjacent blocks: they read the same input rows from L2
  const int r = row0 + blockIdx.y, og = blockIdx.x, tid = threadIdx.x;
  const int sw = s.seg_of_row(r);
  const int fb = s.frame_begin(sw), t = s.frames(sw), ti = r - s.row_begin(sw);
  const int q = tid >> 6, idx = tid & 63;
  const int f0 = (idx & 7) * TP_P, o0 = (idx >> 3) * TP_C;
  // tap c*49 + i*7 + j of a stage reads raw row (i, c) at column f + j + 1 (= x column f+j-3, +4)
  for (int e = tid; e < 2 * CV2_MP; e += TP_THREADS) {
    const int cl = e / 49, rem = e - cl * 49, i = rem / 7, j = rem - i * 7;
    tapoff[e] = (i * CV2_CC + cl) * CV2_RW + j + 1;
  }
  // zeros that no copy overwrites: the pad columns, and whole rows outside the segment
  for (int e = tid; e < CV2_RAW; e += TP_THREADS) {
    const int col = e % CV2_RW, i = e / (CV2_RW * CV2_CC);
    const int tt = ti * 5 + i - 1;
    if (col < 4 || col >= 4 + DIM || tt < 0 || tt >= t) raw[e] = 0.0f;
  }
  const bool w8 = (reinterpret_cast<uintptr_t>(c2) & 7) == 0;
  const bool x16 = (reinterpret_cast<uintptr_t>(y1) & 15) == 0;
  float2 acc[TP_P][TP_C];
#pragma unroll
  for (int p = 0; p < TP_P; p++)
#pragma unroll
    for (int c = 0; c < TP_C; c++) acc[p][c] = make_float2(0.0f, 0.0f);
#pragma unroll 1
  for (int c0 = 0; c0 < C1; c0 += CV2_CC) {
    __syncthreads();  // the previous stage is consumed (and the zeros / offsets are visible)
    for (int e = tid; e < CV2_MP * CV2_CH; e += TP_THREADS) {  // weight pairs from the [out][tap] layout
      const int o = e / CV2_MP, m = e - o * CV2_MP;
      const float* w = c2 + static_cast<int64_t>(og * CV2_CH + o) * K2 + c0 * 49 + 2 * m;
      float2* d = Wt + m * CV2_WS + o;
      if (w8) {
        cp_async8(d, w);
      } else {
        cp_async4(d, w);
        cp_async4(reinterpret_cast<float*>(d) + 1, w + 1);
      }
    }
    for (int e = tid; e < 7 * CV2_CC * (DIM / 4); e += TP_THREADS) {
      const int row = e / (DIM / 4), p4 = e - row * (DIM / 4), i = row / CV2_CC, cl = row - i * CV2_CC;
      const int tt = ti * 5 + i - 1;
      if (tt >= 0 && tt < t) {
        const float* src = y1 + static_cast<int64_t>(fb + tt) * (C1 * DIM) + (c0 + cl) * DIM + 4 * p4;
        float* d = raw + row * CV2_RW + 4 + 4 * p4;
        if (x16) {
          cp_async16(d, src);
        } else {
#pragma unroll
          for (int u = 0; u < 4; u++) cp_async4(d + u, src + u);
        }
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    {  // warp per tap pair, lane per position (the offsets are warp-uniform)
      const int warp = tid >> 5, lane = tid & 31;
      for (int m = warp; m < CV2_MP; m += TP_THREADS / 32) {
        const float* a = raw + tapoff[2 * m];
        const float* b = raw + tapoff[2 * m + 1];
        X2[m * DIM + lane] = make_float2(a[lane], b[lane]);
        if (lane < DIM - 32) X2[m * DIM + 32 + lane] = make_float2(a[32 + lane], b[32 + lane]);
      }
    }
    __syncthreads();
    tp_accumulate<DIM, CV2_WS, 12>(X2, Wt, CV2_MP, (q - (c0 >> 1)) & 3, f0, o0, acc);
  }
  __syncthreads();
  float2* part = reinterpret_cast<float2*>(sm);  // [4][32][42]
#pragma unroll
  for (int p = 0; p < TP_P; p++)
#pragma unroll
    for (int c = 0; c < TP_C; c++) part[(q * CV2_CH + o0 + c) * CV2_PS + f0 + p] = acc[p][c];
  __syncthreads();
  float* out = y2 + static_cast<int64_t>(r) * (C2 * W2) + og * CV2_CH * W2;
  for (int e = tid; e < CV2_CH * DIM; e += TP_THREADS) {
    const int o = e / DIM, f = e - o * DIM;
    out[o * W2 + f] = fmaxf(tp_fold(part, CV2_CH, CV2_PS, o, f), 0.0f);
  }
  if (tid < CV2_CH) out[tid * W2 + DIM] = 0.0f;
}

// Position-pair conv2 (the engine's; weights transposed once per model to c2t[k][o]).  Warp w
// accumulates dotf lane w of every output of the block: the lane's taps k = w, w+8, ... in
// order, which in stage s are the stage taps t = (w - 4s) mod 8, +8, ... (196 = 4 mod 8).  A
// thread owns 4 output channels x 10 positions as 5 packed pairs (f, f+1) of that lane.  The two
// inputs of a position pair at one tap are adjacent in the staged input row, so they are one
// 8-byte load: each stage's input rows are staged twice, the second copy shifted by one float,
// and a tap reads whichever copy puts its pairs on an 8-byte boundary.  A product pair is one
// packed fma.rn(x, w, -0) -- exactly the rounded product, the sign of a zero product included --
// with the -0 a kernel argument, so that the code generator cannot turn it into a multiply and
// contract that with the following packed rounded add; the accumulate is that add.  Every
// element thus rounds exactly like the scalar dotf sequence, at two packed instructions per two
// multiply-adds.  Stages (4 input channels: the weights [196 taps][32 channels]
// and both copies of 7 input rows) are double-buffered by cp.async, one barrier per stage.
constexpr int CP_CH = 32;                          // output channels per block
constexpr int CP_CC = 4;                           // input channels per stage
constexpr int CP_T = CP_CC * 49;                   // taps per stage
constexpr int CP_NST = C1 / CP_CC;                 // stages
constexpr int CP_RW = 48;                          // staged row: 4 zeros | 40 values | 4 zeros
constexpr int CP_RAW = 7 * CP_CC * CP_RW;          // floats of one copy of a stage's input rows
constexpr int CP_BUF = CP_T * CP_CH + 2 * CP_RAW;  // floats of one stage buffer: weights, copy 0, copy 1
constexpr int CP_PS = DIM + 2;                     // row stride of the lane-fold buffer
constexpr int CP_SMEM = cmax(2 * CP_BUF * 4 + CP_T * 4, 8 * CP_CH * CP_PS * 4);
static_assert(CP_NST * CP_CC == C1 && (CP_BUF * 4) % 16 == 0 && (CP_T * CP_CH * 4) % 16 == 0 &&
                  (CP_RAW * 4) % 16 == 0 && CP_T % 8 == 4,
              "position-pair conv2 layout");

__global__ void __launch_bounds__(TP_THREADS, 3) conv2p_k(const float* __restrict__ y1, const float* __restrict__ c2t,
                                                       Segs s, int row0, float* __restrict__ y2, float nz) {
  extern __shared__ __align__(16) float sm[];
  const float2 z2 = make_float2(nz, nz);
  int* tapoff = reinterpret_cast<int*>(sm + 2 * CP_BUF);  // [196] tap -> float offset from copy 0
  const int r = row0 + blockIdx.y, og = blockIdx.x, tid = threadIdx.x;
  const int sw = s.seg_of_row(r);
  const int fb = s.frame_begin(sw), t = s.frames(sw), ti = r - s.row_begin(sw);
  const int lane = tid >> 5, cg = tid & 7, pg = (tid >> 3) & 3;
  const int f0 = 10 * pg, o0 = 4 * cg;
  // tap c*49 + i*7 + j reads row (i, c) at column f + j + 1 of copy 0 (x column f+j-3, +4); for
  // even j the same pair starts at column f + j of copy 1 (copy1[k] = copy0[k + 1]), so that
  // every pair (f even) starts on an 8-byte boundary
  for (int e = tid; e < CP_T; e += TP_THREADS) {
    const int cl = e / 49, rem = e - cl * 49, i = rem / 7, j = rem - i * 7, row = i * CP_CC + cl;
    tapoff[e] = (j & 1) ? row * CP_RW + j + 1 : CP_RAW + row * CP_RW + j;
  }
  // zeros that no copy overwrites, in both buffers: copy 0's columns 0-3 and 44-47, copy 1's
  // 0-2 and 43-47, and whole rows outside the segment
  for (int e = tid; e < 2 * 2 * CP_RAW; e += TP_THREADS) {
    const int b = e / (2 * CP_RAW), cpy = (e / CP_RAW) & 1, w = e % CP_RAW;
    const int col = w % CP_RW, i = w / (CP_RW * CP_CC), tt = ti * 5 + i - 1;
    const int lo = cpy ? 3 : 4;
    if (col < lo || col >= lo + DIM || tt < 0 || tt >= t) sm[b * CP_BUF + CP_T * CP_CH + e % (2 * CP_RAW)] = 0.0f;
  }
  auto load_stage = [&](int st, int b) {
    float* buf = sm + b * CP_BUF;
    const float* src = c2t + static_cast<int64_t>(st) * CP_T * C2 + og * CP_CH;
    for (int e = tid; e < CP_T * (CP_CH / 4); e += TP_THREADS) {
      const int tp = e >> 3, q = e & 7;
      cp_async16(buf + tp * CP_CH + 4 * q, src + tp * C2 + 4 * q);
    }
    float* c0p = buf + CP_T * CP_CH;
    for (int e = tid; e < 7 * CP_CC * (DIM / 4); e += TP_THREADS) {
      const int row = e / (DIM / 4), p4 = e - row * (DIM / 4), i = row / CP_CC, cl = row - i * CP_CC;
      const int tt = ti * 5 + i - 1;
      if (tt >= 0 && tt < t)
        cp_async16(c0p + row * CP_RW + 4 + 4 * p4,
                   y1 + static_cast<int64_t>(fb + tt) * (C1 * DIM) + (st * CP_CC + cl) * DIM + 4 * p4);
    }
    for (int e = tid; e < 7 * CP_CC * DIM; e += TP_THREADS) {
      const int row = e / DIM, c = e - row * DIM, i = row / CP_CC, cl = row - i * CP_CC;
      const int tt = ti * 5 + i - 1;
      if (tt >= 0 && tt < t)
        cp_async4(c0p + CP_RAW + row * CP_RW + 3 + c,
                  y1 + static_cast<int64_t>(fb + tt) * (C1 * DIM) + (st * CP_CC + cl) * DIM + c);
    }
    cp_async_commit();
  };
  load_stage(0, 0);
  float2 acc[5][4];
#pragma unroll
  for (int k = 0; k < 5; k++)
#pragma unroll
    for (int c = 0; c < 4; c++) acc[k][c] = make_float2(0.0f, 0.0f);
#pragma unroll 1
  for (int st = 0; st < CP_NST; st++) {
    cp_async_wait<0>();
    __syncthreads();  // stage st landed everywhere; stage st-1's buffer is consumed
    if (st + 1 < CP_NST) load_stage(st + 1, (st + 1) & 1);
    const float* buf = sm + (st & 1) * CP_BUF;
    const float* xb = buf + CP_T * CP_CH + f0;
    const float* wb = buf + o0;
#pragma unroll 12
    for (int tp = (lane - 4 * st) & 7; tp < CP_T; tp += 8) {
      const float* xr = xb + tapoff[tp];
      float2 xv[5];
#pragma unroll
      for (int k = 0; k < 5; k++) xv[k] = *reinterpret_cast<const float2*>(xr + 2 * k);
      const float4 w4 = *reinterpret_cast<const float4*>(wb + tp * CP_CH);
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int k = 0; k < 5; k++)
#pragma unroll
        for (int c = 0; c < 4; c++)
          acc[k][c] = add2_rn(acc[k][c], fma2_rn(xv[k], make_float2(wv[c], wv[c]), z2));
    }
  }
  __syncthreads();
  float* part = sm;  // [8 lanes][32 channels][42]
#pragma unroll
  for (int k = 0; k < 5; k++)
#pragma unroll
    for (int c = 0; c < 4; c++)
      *reinterpret_cast<float2*>(part + (lane * CP_CH + o0 + c) * CP_PS + f0 + 2 * k) = acc[k][c];
  __syncthreads();
  float* out = y2 + static_cast<int64_t>(r) * (C2 * W2) + og * CP_CH * W2;
  for (int e = tid; e < CP_CH * DIM; e += TP_THREADS) {
    const int o = e / DIM, f = e - o * DIM;
    const float* pp = part + o * CP_PS + f;
    float v = __fadd_rn(pp[0], pp[CP_CH * CP_PS]);
#pragma unroll
    for (int l = 2; l < 8; l++) v = __fadd_rn(v, pp[l * CP_CH * CP_PS]);
    out[o * W2 + f] = fmaxf(v, 0.0f);
  }
  if (tid < CP_CH) out[tid * W2 + DIM] = 0.0f;
}

// y3[r][o*20+f] = relu(dotf(c3[o], patch)), patch[c*9+i*3+j] = y2[r+i-1][c][2f+j] (zero
// outside the segment) -- src/model.rs:446-468.  Block = (row r, 64 output channels);
// stages of 8 input channels.
__global__ void __launch_bounds__(TP_THREADS, 3) conv3_k(const float* __restrict__ y2, const float* __restrict__ c3,
                                                      Segs s, int row0, float* __restrict__ y3) {
  extern __shared__ __align__(16) float sm[];
  float2* X2 = reinterpret_cast<float2*>(sm);    // [36][20]
  float2* Wt = X2 + CV3_MP * 20;                  // [36][66]
  float* raw = reinterpret_cast<float*>(Wt + CV3_MP * CV3_WS);  // [3 rows][16 channels][41]
  int* tapoff = reinterpret_cast<int*>(raw + CV3_RAW);          // [72] tap -> raw offset (+ 2f)
  // the channel groups of a row are adjacent blocks: they read the same input rows from L2
  const int r = row0 + blockIdx.y, og = blockIdx.x, tid = threadIdx.x;
  const int sw = s.seg_of_row(r);
  const int rb = s.row_begin(sw), t1 = s.rows(sw), ti = r - rb;
  const int q = tid >> 6, idx = tid & 63;
  const int f0 = (idx & 3) * TP_P, o0 = (idx >> 2) * TP_C;
  // tap c*9 + i*3 + j of a stage reads raw row (i, c) at column 2f + j
  for (int e = tid; e < 2 * CV3_MP; e += TP_THREADS) {
    const int cl = e / 9, rem = e - cl * 9, i = rem / 3, j = rem - i * 3;
    tapoff[e] = (i * CV3_CC + cl) * CV3_RW + j;
  }
  for (int e = tid; e < CV3_RAW; e += TP_THREADS) {  // rows outside the segment stay zero
    const int i = e / (CV3_RW * CV3_CC), tt = ti + i - 1;
    if (tt < 0 || tt >= t1) raw[e] = 0.0f;
  }
  const bool w8 = (reinterpret_cast<uintptr_t>(c3) & 7) == 0;
  const bool y16 = (reinterpret_cast<uintptr_t>(y2) & 15) == 0;
  float2 acc[TP_P][TP_C];
#pragma unroll
  for (int p = 0; p < TP_P; p++)
#pragma unroll
    for (int c = 0; c < TP_C; c++) acc[p][c] = make_float2(0.0f, 0.0f);
#pragma unroll 1
  for (int c0 = 0; c0 < C2; c0 += CV3_CC) {
    __syncthreads();
    for (int e = tid; e < CV3_MP * CV3_CH; e += TP_THREADS) {  // weight pairs from the [out][tap] layout
      const int o = e / CV3_MP, m = e - o * CV3_MP;
      const float* w = c3 + static_cast<int64_t>(og * CV3_CH + o) * K3 + c0 * 9 + 2 * m;
      float2* d = Wt + m * CV3_WS + o;
      if (w8) {
        cp_async8(d, w);
      } else {
        cp_async4(d, w);
        cp_async4(reinterpret_cast<float*>(d) + 1, w + 1);
      }
    }
    for (int i = 0; i < 3; i++) {  // input row i: channels c0 .. c0+15 are 656 contiguous floats
      const int tt = ti + i - 1;
      if (tt < 0 || tt >= t1) continue;  // block-uniform; the row stays zero
      const float* src = y2 + static_cast<int64_t>(rb + tt) * (C2 * W2) + c0 * W2;
      float* dst = raw + i * CV3_CC * CV3_RW;
      if (y16) {
        for (int e = tid; e < CV3_CC * W2 / 4; e += TP_THREADS) cp_async16(dst + 4 * e, src + 4 * e);
      } else {
        for (int e = tid; e < CV3_CC * W2; e += TP_THREADS) cp_async4(dst + e, src + e);
      }
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    {  // warp per tap pair, lane per position
      const int warp = tid >> 5, lane = tid & 31;
      for (int m = warp; m < CV3_MP; m += TP_THREADS / 32)
        if (lane < 20) X2[m * 20 + lane] = make_float2(raw[tapoff[2 * m] + 2 * lane], raw[tapoff[2 * m + 1] + 2 * lane]);
    }
    __syncthreads();
    tp_accumulate<20, CV3_WS, 4>(X2, Wt, CV3_MP, (q - (c0 >> 1)) & 3, f0, o0, acc);
  }
  __syncthreads();
  float2* part = reinterpret_cast<float2*>(sm);  // [4][64][21]
#pragma unroll
  for (int p = 0; p < TP_P; p++)
#pragma unroll
    for (int c = 0; c < TP_C; c++) part[(q * CV3_CH + o0 + c) * CV3_PS + f0 + p] = acc[p][c];
  __syncthreads();
  float* out = y3 + static_cast<int64_t>(r) * FLAT + og * CV3_CH * 20;
  for (int e = tid; e < CV3_CH * 20; e += TP_THREADS) {
    const int o = e / 20, f = e - o * 20;
    out[o * 20 + f] = fmaxf(tp_fold(part, CV3_CH, CV3_PS, o, f), 0.0f);
  }
}

// ------------------------------------------------------------------------ quant
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// per-row dynamic quant (src/kernels.rs:11-25): one warp per row.  The max is order-free,
// every element's rounding is independent, so any split is exact.
__global__ void __launch_bounds__(256) quant_rows_k(const float* __restrict__ x, int m, int k, int ldx,
                                                    const unsigned* __restrict__ rowmax, int8_t* __restrict__ xq,
                                                    float* __restrict__ xs) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= m) return;
  const float* r = x + static_cast<int64_t>(row) * ldx;
  const bool vec = ((k & 3) == 0) && ((reinterpret_cast<uintptr_t>(r) & 15) == 0);
  if (k == D && vec && !rowmax) {  // the engine's rows: held in registers, one pass, loads all in flight
    float4 v[4];
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = *reinterpret_cast<const float4*>(r + lane * 4 + 128 * i);
    float m4 = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) m4 = fmaxf(m4, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    m4 = warp_max(m4);
    const float sc4 = quant_scale(m4), inv4 = quant_inv(sc4);
    int8_t* q4 = xq + static_cast<int64_t>(row) * k;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      char4 c;
      c.x = quant_one(v[i].x, inv4); c.y = quant_one(v[i].y, inv4); c.z = quant_one(v[i].z, inv4); c.w = quant_one(v[i].w, inv4);
      *reinterpret_cast<char4*>(q4 + lane * 4 + 128 * i) = c;
    }
    if (lane == 0) xs[row] = sc4;
    return;
  }
  float mx;
  if (rowmax) {
    mx = __uint_as_float(rowmax[row]);
  } else {
    mx = 0.0f;
    if (vec) {
      for (int j = lane * 4; j < k; j += 128) {
        const float4 v = *reinterpret_cast<const float4*>(r + j);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
    } else {
      for (int j = lane; j < k; j += 32) mx = fmaxf(mx, fabsf(r[j]));
    }
    mx = warp_max(mx);
  }
  const float sc = quant_scale(mx), inv = quant_inv(sc);
  int8_t* q = xq + static_cast<int64_t>(row) * k;
  if (vec) {
    for (int j = lane * 4; j < k; j += 128) {
      const float4 v = *reinterpret_cast<const float4*>(r + j);
      char4 c;
      c.x = quant_one(v.x, inv); c.y = quant_one(v.y, inv); c.z = quant_one(v.z, inv); c.w = quant_one(v.w, inv);
      *reinterpret_cast<char4*>(q + j) = c;
    }
  } else {
    for (int j = lane; j < k; j += 32) q[j] = quant_one(r[j], inv);
  }
  if (lane == 0) xs[row] = sc;
}

// ------------------------------------------------------------------------ LayerNorm + quant
// src/model.rs:693-704 (+ the residual add of :493 / csrc/wtl_kern.cu:170-216 when o != 0).
// Mean and variance are sequential left folds on the CPU, i.e. chains of 512 dependent
// rounded adds per row, so a block keeps 128 rows folding at once: the rows stream through
// shared memory in column chunks (coalesced cp.async, three chunks in flight), and thread i folds row
// i over each chunk in column order -- pass 1 the sum, pass 2 the squared deviations.  Then 16
// warps normalise, write the residual and quantise one row each at a time, coalesced, with
// gamma / beta in registers.  The residual h + o is recomputed wherever it is needed (the same
// rounded add every time).
constexpr int LN_ROWS = 128;
constexpr int LN_THREADS = 512;
template <bool RES>
struct LnCfg {
  static constexpr int CW = RES ? 32 : 64;   // columns per chunk
  static constexpr int NCH = D / CW;         // chunks per pass
  static constexpr int RS = CW + 4;          // shared row stride in floats (conflict-free float4 rows)
  static constexpr int NSRC = RES ? 2 : 1;   // h (+ o)
  static constexpr int NBUF = 4;             // chunks in flight: 3 loading while one is folded
  static constexpr int BUF = NSRC * LN_ROWS * RS;
  static constexpr int SMEM = NBUF * BUF * 4 + 2 * LN_ROWS * 4;
};

__device__ __forceinline__ float4 add4_rn(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

template <bool RES>
__global__ void __launch_bounds__(LN_THREADS) ln_quant_k(float* __restrict__ h, const float* __restrict__ o,
                                                         const float* __restrict__ g, const float* __restrict__ b,
                                                         int m, int8_t* __restrict__ xq, float* __restrict__ xs) {
  using C = LnCfg<RES>;
  extern __shared__ __align__(16) float sm[];
  float* mean = sm + C::NBUF * C::BUF;
  float* rinv = mean + LN_ROWS;
  const int r0 = blockIdx.x * LN_ROWS;
  const int nr = min(LN_ROWS, m - r0);
  const int tid = threadIdx.x;
  constexpr int NK = 2 * C::NCH;  // chunks of both passes
  // chunk k (0 .. NK-1) -> buffer k % NBUF; one commit group per chunk (empty past the end)
  auto load = [&](int k) {
    if (k < NK) {
      float* dst = sm + (k % C::NBUF) * C::BUF;
      const int col0 = (k % C::NCH) * C::CW;
      for (int e = tid; e < nr * (C::CW / 4); e += LN_THREADS) {
        const int rr = e / (C::CW / 4), c4 = e - rr * (C::CW / 4);
        const int64_t src = static_cast<int64_t>(r0 + rr) * D + col0 + 4 * c4;
        cp_async16(dst + rr * C::RS + 4 * c4, h + src);
        if constexpr (RES) cp_async16(dst + LN_ROWS * C::RS + rr * C::RS + 4 * c4, o + src);
      }
    }
    cp_async_commit();
  };
  for (int k = 0; k < C::NBUF - 1; k++) load(k);
  float sum = 0.0f, s2 = 0.0f, mu = 0.0f;
#pragma unroll 1
  for (int k = 0; k < NK; k++) {
    cp_async_wait<C::NBUF - 2>();  // chunk k has landed (the next NBUF-2 may still be loading)
    __syncthreads();               // ... for every thread; chunk k-1's buffer is free again
    load(k + C::NBUF - 1);
    if (tid < nr) {
      const float4* hr = reinterpret_cast<const float4*>(sm + (k % C::NBUF) * C::BUF + tid * C::RS);
      const float4* orow = reinterpret_cast<const float4*>(sm + (k % C::NBUF) * C::BUF + LN_ROWS * C::RS + tid * C::RS);
      if (k < C::NCH) {
#pragma unroll 8
        for (int c = 0; c < C::CW / 4; c++) {
          float4 v = hr[c];
          if constexpr (RES) v = add4_rn(v, orow[c]);
          sum = __fadd_rn(sum, v.x);
          sum = __fadd_rn(sum, v.y);
          sum = __fadd_rn(sum, v.z);
          sum = __fadd_rn(sum, v.w);
        }
        if (k == C::NCH - 1) mu = __fdiv_rn(sum, static_cast<float>(D));
      } else {
#pragma unroll 8
        for (int c = 0; c < C::CW / 4; c++) {
          float4 v = hr[c];
          if constexpr (RES) v = add4_rn(v, orow[c]);
          const float dx = __fsub_rn(v.x, mu), dy = __fsub_rn(v.y, mu), dz = __fsub_rn(v.z, mu),
                      dw = __fsub_rn(v.w, mu);
          s2 = __fadd_rn(s2, __fmul_rn(dx, dx));
          s2 = __fadd_rn(s2, __fmul_rn(dy, dy));
          s2 = __fadd_rn(s2, __fmul_rn(dz, dz));
          s2 = __fadd_rn(s2, __fmul_rn(dw, dw));
        }
      }
    }
  }
  cp_async_wait<0>();
  if (tid < nr) {
    const float var = __fdiv_rn(s2, static_cast<float>(D));
    mean[tid] = mu;
    rinv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-6f)));
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  float4 gg[4], bb[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    gg[k] = __ldg(reinterpret_cast<const float4*>(g) + lane + 32 * k);
    bb[k] = __ldg(reinterpret_cast<const float4*>(b) + lane + 32 * k);
  }
  // rows rr = warp, warp + 16, ...: the next row's values load while this row is computed
  float4 nh[4], no[4];
  auto fetch = [&](int rr) {
    const float4* hr = reinterpret_cast<const float4*>(h + static_cast<int64_t>(r0 + rr) * D);
#pragma unroll
    for (int k = 0; k < 4; k++) nh[k] = hr[lane + 32 * k];
    if constexpr (RES) {
      const float4* orow = reinterpret_cast<const float4*>(o + static_cast<int64_t>(r0 + rr) * D);
#pragma unroll
      for (int k = 0; k < 4; k++) no[k] = orow[lane + 32 * k];
    }
  };
  if (warp < nr) fetch(warp);
  for (int rr = warp; rr < nr; rr += LN_THREADS / 32) {
    const float mu_r = mean[rr], iv = rinv[rr];
    float4* hr = reinterpret_cast<float4*>(h + static_cast<int64_t>(r0 + rr) * D);
    float4 ch[4], co[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      ch[k] = nh[k];
      co[k] = no[k];
    }
    if (rr + LN_THREADS / 32 < nr) fetch(rr + LN_THREADS / 32);
    float4 y[4];
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      float4 v = ch[k];
      if constexpr (RES) {
        v = add4_rn(v, co[k]);
        hr[lane + 32 * k] = v;
      }
      y[k].x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, mu_r), iv), gg[k].x), bb[k].x);
      y[k].y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, mu_r), iv), gg[k].y), bb[k].y);
      y[k].z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, mu_r), iv), gg[k].z), bb[k].z);
      y[k].w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, mu_r), iv), gg[k].w), bb[k].w);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(y[k].x), fabsf(y[k].y)), fmaxf(fabsf(y[k].z), fabsf(y[k].w))));
    }
    mx = warp_max(mx);
    const float sc = quant_scale(mx), inv = quant_inv(sc);
    char4* q = reinterpret_cast<char4*>(xq + static_cast<int64_t>(r0 + rr) * D);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      char4 c;
      c.x = quant_one(y[k].x, inv); c.y = quant_one(y[k].y, inv); c.z = quant_one(y[k].z, inv); c.w = quant_one(y[k].w, inv);
      q[lane + 32 * k] = c;
    }
    if (lane == 0) xs[r0 + rr] = sc;
  }
}

// LayerNorm + quant without a residual (the engine's case: the GEMM epilogue already added
// it), with the block's rows resident in shared memory: 56 rows of 512 floats, loaded once by
// cp.async in 8 column chunks (one commit group each).  Thread r < 56 folds row r's sum while
// the chunks land, then its squared deviations from shared memory (the same left folds as
// ln_quant_k); 8 warps then normalise and quantise the rows from shared memory.  Float4 slot
// c4 of row r sits at slot c4 ^ (r & 7), so the 8 rows a quarter-warp folds at one column hit
// distinct banks and a warp's 32 consecutive slots of one row stay conflict-free.  Two blocks
// (2 x 115 KB) fit an SM, so 16384 rows are one wave of 293 blocks.
constexpr int LR_ROWS = 56;
constexpr int LR_THREADS = 256;
constexpr size_t LR_SMEM = static_cast<size_t>(LR_ROWS) * D * 4 + 2 * LR_ROWS * 4;
__device__ __forceinline__ int lr_slot(int r, int c4) { return r * (D / 4) + (c4 ^ (r & 7)); }
__device__ __forceinline__ void cp_async_wait_n(int n) {  // n in 0..7, a run-time count
  switch (n) {
    case 7: cp_async_wait<7>(); break;
    case 6: cp_async_wait<6>(); break;
    case 5: cp_async_wait<5>(); break;
    case 4: cp_async_wait<4>(); break;
    case 3: cp_async_wait<3>(); break;
    case 2: cp_async_wait<2>(); break;
    case 1: cp_async_wait<1>(); break;
    default: cp_async_wait<0>(); break;
  }
}

// rpb <= LR_ROWS rows per block (the launcher sizes it so that a small M still fills the GPU)
__global__ void __launch_bounds__(LR_THREADS, 2) ln_rows_k(const float* __restrict__ h, const float* __restrict__ g,
                                                           const float* __restrict__ b, int m, int rpb,
                                                           int8_t* __restrict__ xq, float* __restrict__ xs) {
  extern __shared__ __align__(16) float sm[];
  float4* S = reinterpret_cast<float4*>(sm);
  float* mean = sm + rpb * D;
  float* rinv = mean + rpb;
  const int r0 = blockIdx.x * rpb, nr = min(rpb, m - r0), tid = threadIdx.x;
  for (int c = 0; c < 8; c++) {  // chunk c: columns 64c .. 64c+63 of every row
    for (int e = tid; e < nr * 16; e += LR_THREADS) {
      const int rr = e >> 4, c4 = 16 * c + (e & 15);
      cp_async16(S + lr_slot(rr, c4), h + static_cast<int64_t>(r0 + rr) * D + 4 * c4);
    }
    cp_async_commit();
  }
  // the folds are chains of dependent adds: each chunk's loads are all issued before its adds
  float sum = 0.0f;
  for (int c = 0; c < 8; c++) {
    cp_async_wait_n(7 - c);  // this thread's copies of chunk c have landed ...
    __syncthreads();         // ... and every thread's
    if (tid < nr) {
      float4 v[16];
#pragma unroll
      for (int k = 0; k < 16; k++) v[k] = S[lr_slot(tid, 16 * c + k)];
#pragma unroll
      for (int k = 0; k < 16; k++) {
        sum = __fadd_rn(sum, v[k].x);
        sum = __fadd_rn(sum, v[k].y);
        sum = __fadd_rn(sum, v[k].z);
        sum = __fadd_rn(sum, v[k].w);
      }
    }
  }
  if (tid < nr) {
    const float mu = __fdiv_rn(sum, static_cast<float>(D));
    float s2 = 0.0f;
    float4 cur[8], nxt[8];
#pragma unroll
    for (int k = 0; k < 8; k++) cur[k] = S[lr_slot(tid, k)];
#pragma unroll 1
    for (int c4 = 0; c4 < D / 4; c4 += 8) {
      if (c4 + 8 < D / 4) {
#pragma unroll
        for (int k = 0; k < 8; k++) nxt[k] = S[lr_slot(tid, c4 + 8 + k)];
      }
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const float4 v = cur[k];
        const float dx = __fsub_rn(v.x, mu), dy = __fsub_rn(v.y, mu), dz = __fsub_rn(v.z, mu), dw = __fsub_rn(v.w, mu);
        s2 = __fadd_rn(s2, __fmul_rn(dx, dx));
        s2 = __fadd_rn(s2, __fmul_rn(dy, dy));
        s2 = __fadd_rn(s2, __fmul_rn(dz, dz));
        s2 = __fadd_rn(s2, __fmul_rn(dw, dw));
      }
#pragma unroll
      for (int k = 0; k < 8; k++) cur[k] = nxt[k];
    }
    mean[tid] = mu;
    rinv[tid] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s2, static_cast<float>(D)), 1e-6f)));
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  float4 gg[4], bb[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    gg[k] = __ldg(reinterpret_cast<const float4*>(g) + lane + 32 * k);
    bb[k] = __ldg(reinterpret_cast<const float4*>(b) + lane + 32 * k);
  }
  // four rows per step (rr + 8a; rows past the end repeat rr, writing the same values), so
  // the four reductions and quantisations overlap
  constexpr int NB = 4, NW = LR_THREADS / 32;
  for (int rr = warp; rr < nr; rr += NB * NW) {
    int row[NB];
#pragma unroll
    for (int a = 0; a < NB; a++) row[a] = rr + a * NW < nr ? rr + a * NW : rr;
    float4 y[NB][4];
    float mx[NB];
#pragma unroll
    for (int a = 0; a < NB; a++) {
      const float mu_r = mean[row[a]], iv = rinv[row[a]];
      mx[a] = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float4 v = S[lr_slot(row[a], lane + 32 * k)];
        y[a][k].x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, mu_r), iv), gg[k].x), bb[k].x);
        y[a][k].y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, mu_r), iv), gg[k].y), bb[k].y);
        y[a][k].z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, mu_r), iv), gg[k].z), bb[k].z);
        y[a][k].w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, mu_r), iv), gg[k].w), bb[k].w);
        mx[a] = fmaxf(mx[a], fmaxf(fmaxf(fabsf(y[a][k].x), fabsf(y[a][k].y)), fmaxf(fabsf(y[a][k].z), fabsf(y[a][k].w))));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
      for (int a = 0; a < NB; a++) mx[a] = fmaxf(mx[a], __shfl_xor_sync(0xffffffffu, mx[a], o));
#pragma unroll
    for (int a = 0; a < NB; a++) {
      const float sc = quant_scale(mx[a]), inv = quant_inv(sc);
      char4* q = reinterpret_cast<char4*>(xq + static_cast<int64_t>(r0 + row[a]) * D);
#pragma unroll
      for (int k = 0; k < 4; k++) {
        char4 cq;
        cq.x = quant_one(y[a][k].x, inv); cq.y = quant_one(y[a][k].y, inv);
        cq.z = quant_one(y[a][k].z, inv); cq.w = quant_one(y[a][k].w, inv);
        q[lane + 32 * k] = cq;
      }
      if (lane == 0) xs[r0 + row[a]] = sc;
    }
  }
}

// LayerNorm for any d (the reference ABI takes d as an argument): one block per row,
// thread 0 folds like the CPU.  Used only when d != 512.
__global__ void __launch_bounds__(256) ln_quant_any_k(float* __restrict__ h, const float* __restrict__ o,
                                                      const float* __restrict__ g, const float* __restrict__ b,
                                                      int d, int8_t* __restrict__ xq, float* __restrict__ xs) {
  __shared__ float st[2];
  __shared__ float red[8];
  float* x = h + static_cast<int64_t>(blockIdx.x) * d;
  if (o) {
    const float* oo = o + static_cast<int64_t>(blockIdx.x) * d;
    for (int j = threadIdx.x; j < d; j += blockDim.x) x[j] = __fadd_rn(x[j], oo[j]);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int j = 0; j < d; j++) sum = __fadd_rn(sum, x[j]);
    const float mu = __fdiv_rn(sum, static_cast<float>(d));
    float s2 = 0.0f;
    for (int j = 0; j < d; j++) {
      const float dd = __fsub_rn(x[j], mu);
      s2 = __fadd_rn(s2, __fmul_rn(dd, dd));
    }
    st[0] = mu;
    st[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s2, static_cast<float>(d)), 1e-6f)));
  }
  __syncthreads();
  const float mu = st[0], iv = st[1];
  float mx = 0.0f;
  for (int j = threadIdx.x; j < d; j += blockDim.x)
    mx = fmaxf(mx, fabsf(__fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x[j], mu), iv), g[j]), b[j])));
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < (blockDim.x >> 5); w++) mx = fmaxf(mx, red[w]);
  const float sc = quant_scale(mx), inv = quant_inv(sc);
  for (int j = threadIdx.x; j < d; j += blockDim.x)
    xq[static_cast<int64_t>(blockIdx.x) * d + j] =
        quant_one(__fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x[j], mu), iv), g[j]), b[j]), inv);
  if (threadIdx.x == 0) xs[blockIdx.x] = sc;
}

// ------------------------------------------------------------------------ conv3 + certified quant
// The engine's conv3: y3 feeds only its row's int8 quantisation (src/model.rs:489,
// quant(y3, FLAT)), so the kernel computes y3 with fused multiply-adds in any order, bounds
// the difference to the reference's dotf result, and quantises exactly as in quant, taking
// the row maximum and every element near a rounding boundary from the reference-order value
// (the same reasoning as the certified GELU).
//
// Bound.  For output (o, f) with patch a and weight row w, both sums are the exact sum with term
// k multiplied by at most n(k) factors (1 + d), |d| <= u = 2^-24: in the dotf order its product,
// the adds of its lane chain from chunk c = k / 8 on (72 - c) and the lane fold (7 for lanes 0
// and 1, 8 - l for lane l >= 2); in the fused multiply-add order the stage chain from tap
// i = k % 36 on (36 - i) and the adds of the stage partials into the total (15 for stage 0,
// 16 - s for stage s >= 1).  Both n <= 131, so each sum is within u (1 + 2^-10) sum_k
// |a_k w_k| n(k) of the exact sum, relu is 1-Lipschitz, and by Cauchy-Schwarz
// |y~ - y| <= E = C3C_BOUND * na(f) * nw(o), with na >= |a|_2 and nw >= |w o n|_2 (the weight
// row scaled by the two depths, computed once per model).
//
// Work split: a block owns 4 output rows (80 positions) and all 192 channels, 16 stages of 4
// input channels (36 taps).  Per stage the weights [36 taps][192] (pre-transposed once per model)
// and the 6 input rows' 4 channels stream in by cp.async (double-buffered), the im2col tile
// P[36][80] is built in shared memory, and thread (cg, pg) < 240 accumulates channels
// {4cg+a, 96+4cg+a} x positions {4pg+b, 40+4pg+b} (a, b < 4) from two 16-byte loads of each.
// Epilogue: the 6 input rows are staged whole for the reference-order values, then per row the
// maximum candidates (y~ + E >= max(y~ - E)) and the near-boundary elements are evaluated in
// dotf order by groups of 8 threads (one per dotf lane, folded in lane order).
constexpr int C3C_R = 4;                 // output rows per block
constexpr int C3C_N = C3C_R * 20;        // positions per block
constexpr int C3C_CC = 4;                // input channels per stage
constexpr int C3C_KS = C3C_CC * 9;       // taps per stage
constexpr int C3C_NST = C2 / C3C_CC;     // stages
constexpr int C3C_RAWR = C3C_CC * W2;    // floats of one staged input row (4 channels x 41)
constexpr int C3C_IN = C3C_R + 2;        // input rows per block
constexpr int C3C_THREADS = 256;
constexpr int C3C_CAP = 2048;            // entries of the reference-order list
constexpr int C3C_YROW = C2 * W2;        // floats of one y2 row (2624)
// shared-memory layout, in floats
constexpr int C3C_OFF_W = 0;                                      // [2][36][192]
constexpr int C3C_OFF_RAW = C3C_OFF_W + 2 * C3C_KS * C3;          // [2][6][164]
constexpr int C3C_OFF_P = C3C_OFF_RAW + 2 * C3C_IN * C3C_RAWR;    // [36][80]
constexpr int C3C_OFF_Q = C3C_OFF_P + C3C_KS * C3C_N;             // int8 [4][3840]
constexpr int C3C_OFF_LIST = C3C_OFF_Q + C3C_R * FLAT / 4;        // int [cap] + float [cap]
constexpr int C3C_OFF_KO = C3C_OFF_LIST + 2 * C3C_CAP;            // int [576]: (i << 16) | (i * 2624 + c * 41 + j)
constexpr int C3C_OFF_NA = C3C_OFF_KO + K3;                       // [80]
constexpr int C3C_OFF_NW = C3C_OFF_NA + C3C_N;                    // [192]
constexpr int C3C_OFF_MISC = C3C_OFF_NW + C3;                     // ints: valid[12], L[4], M[4], cnt, ovf
constexpr int C3C_SMEM = (C3C_OFF_MISC + 32) * 4;
static_assert(C3C_IN * C3C_YROW <= C3C_OFF_P, "the staged y2 rows reuse the weight / raw buffers");
// u (1 + 2^-10): the first-order bound above with margin for its (1 + u)^n - 1 <= n u (1 + n u)
constexpr float C3C_BOUND = 0x1p-24f * (1.0f + 0x1p-10f);

// lane l's dotf chain (taps l, l+8, ..., l+568) of output (row rho, channel o, position f) from
// the staged y2 rows; valid[rho*3 + i] says whether input row rho+i-1 is inside the segment
__device__ __forceinline__ float c3c_lane(const float* y2s, const float* __restrict__ c3, const int* ko,
                                          const int* valid, int rho, int o, int f, int l) {
  const float* wr = c3 + static_cast<int64_t>(o) * K3;
  const float* base = y2s + rho * C3C_YROW + 2 * f;
  float acc = 0.0f;
#pragma unroll 8
  for (int c = 0; c < K3 / 8; c++) {
    const int k = 8 * c + l, e = ko[k];
    const float a = valid[rho * 3 + (e >> 16)] ? base[e & 0xffff] : 0.0f;
    acc = __fadd_rn(acc, __fmul_rn(__ldg(wr + k), a));
  }
  return acc;
}
// fold the 8 lanes of a group in lane order and apply relu (every lane of the group gets it)
__device__ __forceinline__ float c3c_fold(float v) {
  float s = __fadd_rn(__shfl_sync(0xffffffffu, v, 0, 8), __shfl_sync(0xffffffffu, v, 1, 8));
#pragma unroll
  for (int l = 2; l < 8; l++) s = __fadd_rn(s, __shfl_sync(0xffffffffu, v, l, 8));
  return fmaxf(s, 0.0f);
}

// Thread (cg, pg)'s 64 outputs: element j = 8a + b is channel o(a), position n(b); the running
// totals of a stage's partial sums live in tensor memory (this thread's TMEM lane, columns
// 64 (warp / 4) + j), which leaves the registers to the stage accumulators so that two blocks
// fit an SM.
__device__ __forceinline__ int c3c_o(int cg, int a) { return (a < 4 ? 0 : 96) + 4 * cg + (a & 3); }
__device__ __forceinline__ int c3c_n(int pg, int b) { return (b < 4 ? 0 : 40) + 4 * pg + (b & 3); }

__global__ void __launch_bounds__(C3C_THREADS, 2) conv3_cert_k(const float* __restrict__ y2,
                                                              const float* __restrict__ c3,
                                                              const float* __restrict__ c3t,
                                                              const float* __restrict__ nw_g, Segs s, int total,
                                                              int8_t* __restrict__ xq, float* __restrict__ xs) {
  extern __shared__ __align__(16) float sm[];
  float* Wst = sm + C3C_OFF_W;
  float* raw = sm + C3C_OFF_RAW;
  float* P = sm + C3C_OFF_P;
  int8_t* qo = reinterpret_cast<int8_t*>(sm + C3C_OFF_Q);
  int* lst = reinterpret_cast<int*>(sm + C3C_OFF_LIST);
  float* lval = sm + C3C_OFF_LIST + C3C_CAP;
  int* ko = reinterpret_cast<int*>(sm + C3C_OFF_KO);
  float* na = sm + C3C_OFF_NA;
  float* nw = sm + C3C_OFF_NW;
  int* misc = reinterpret_cast<int*>(sm + C3C_OFF_MISC);
  int* valid = misc;                       // [12]
  float* rowL = sm + C3C_OFF_MISC + 12;    // [4]
  float* rowM = sm + C3C_OFF_MISC + 16;    // [4]
  int* cnt = misc + 20;
  int* ovf = misc + 21;
  float* rowInv = sm + C3C_OFF_MISC + 24;  // [4]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(misc + 28);
  const int t = threadIdx.x, warp = t >> 5, r0 = blockIdx.x * C3C_R;
  if (warp == 0) {
    tmem_alloc(tslot, 128);
    tmem_relinquish();
  }
  if (t < 12) {
    const int rho = t / 3, i = t % 3, r = r0 + rho;
    bool ok = false;
    if (r < total) {
      const int w = s.seg_of_row(r), tt = r - s.row_begin(w) + i - 1;
      ok = tt >= 0 && tt < s.rows(w);
    }
    valid[t] = ok;
  }
  if (t < C3C_R) rowL[t] = 0.0f, rowM[t] = 0.0f;
  if (t == 0) *cnt = 0, *ovf = 0;
  for (int k = t; k < K3; k += C3C_THREADS) {
    const int c = k / 9, tap = k - 9 * c, i = tap / 3, j = tap - 3 * i;
    ko[k] = (i << 16) | (i * C3C_YROW + c * W2 + j);
  }
  for (int o = t; o < C3; o += C3C_THREADS) nw[o] = nw_g[o];
  auto load_stage = [&](int st, int buf) {
    const float4* src = reinterpret_cast<const float4*>(c3t + static_cast<int64_t>(st) * C3C_KS * C3);
    float4* dst = reinterpret_cast<float4*>(Wst + buf * C3C_KS * C3);
    for (int e = t; e < C3C_KS * C3 / 4; e += C3C_THREADS) cp_async16(dst + e, src + e);
    for (int e = t; e < C3C_IN * (C3C_RAWR / 4); e += C3C_THREADS) {
      const int ri = e / (C3C_RAWR / 4), q = e - ri * (C3C_RAWR / 4), g = r0 - 1 + ri;
      if (g >= 0 && g < total)
        cp_async16(raw + (buf * C3C_IN + ri) * C3C_RAWR + 4 * q,
                   y2 + static_cast<int64_t>(g) * C3C_YROW + st * C3C_RAWR + 4 * q);
    }
    cp_async_commit();
  };
  load_stage(0, 0);
  const bool act = t < 240;
  const int cg = t % 24, pg = t / 24;
  tc_fence_before();
  __syncthreads();  // valid[], the TMEM address
  tc_fence_after();
  const uint32_t tcol = *tslot + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + static_cast<uint32_t>(64 * (warp >> 2));
  // the im2col tile's source offsets in a stage's raw rows are the same in every stage: this
  // thread's elements e = t + 256 m of P, -1 where the input row lies outside the segment
  constexpr int PB = (C3C_KS * C3C_N + C3C_THREADS - 1) / C3C_THREADS;
  int poff[PB];
#pragma unroll
  for (int m = 0; m < PB; m++) {
    const int e = t + C3C_THREADS * m;
    const int kk = e / C3C_N, n = e - kk * C3C_N, rho = n / 20, f = n - 20 * rho;
    const int cl = kk / 9, tap = kk - 9 * cl, i = tap / 3, j = tap - 3 * i;
    poff[m] = (e < C3C_KS * C3C_N && valid[rho * 3 + i]) ? (rho + i) * C3C_RAWR + cl * W2 + 2 * f + j : -1;
  }
#pragma unroll 1
  for (int st = 0; st < C3C_NST; st++) {
    cp_async_wait<0>();
    __syncthreads();  // stage st visible; the previous stage's P and buffers consumed
    if (st + 1 < C3C_NST) load_stage(st + 1, (st + 1) & 1);
    const float* rw = raw + (st & 1) * C3C_IN * C3C_RAWR;
#pragma unroll
    for (int m = 0; m < PB; m++) {
      const int e = t + C3C_THREADS * m;
      if (e < C3C_KS * C3C_N) P[e] = poff[m] >= 0 ? rw[poff[m]] : 0.0f;
    }
    __syncthreads();
    // accumulators in packed pairs: acc[a][q] = (channel a, positions 2q, 2q+1 of the thread's 8)
    float2 acc[8][4];
#pragma unroll
    for (int a = 0; a < 8; a++)
#pragma unroll
      for (int q = 0; q < 4; q++) acc[a][q] = make_float2(0.0f, 0.0f);
    if (act) {
      const float* wb = Wst + (st & 1) * C3C_KS * C3 + 4 * cg;
      const float* pb = P + 4 * pg;
#pragma unroll 12
      for (int kk = 0; kk < C3C_KS; kk++) {
        const float4 w0 = *reinterpret_cast<const float4*>(wb + kk * C3);
        const float4 w1 = *reinterpret_cast<const float4*>(wb + kk * C3 + 96);
        const float4 p0 = *reinterpret_cast<const float4*>(pb + kk * C3C_N);
        const float4 p1 = *reinterpret_cast<const float4*>(pb + kk * C3C_N + 40);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const float2 pv[4] = {make_float2(p0.x, p0.y), make_float2(p0.z, p0.w), make_float2(p1.x, p1.y),
                              make_float2(p1.z, p1.w)};
#pragma unroll
        for (int a = 0; a < 8; a++) {
          const float2 wd = make_float2(wv[a], wv[a]);
#pragma unroll
          for (int q = 0; q < 4; q++) acc[a][q] = fma2_rn(wd, pv[q], acc[a][q]);
        }
      }
    }
    // running totals (whole warps: tcgen05 ld / st are warp-collective)
#pragma unroll
    for (int h = 0; h < 2; h++) {
      uint32_t r[32];
      if (st > 0) {
        tmem_st_wait();
        tmem_ld32(tcol + 32 * h, r);
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int q = 0; q < 4; q++) {
            const float2 tv = add2_rn(make_float2(__uint_as_float(r[8 * a + 2 * q]), __uint_as_float(r[8 * a + 2 * q + 1])),
                                      acc[4 * h + a][q]);
            r[8 * a + 2 * q] = __float_as_uint(tv.x), r[8 * a + 2 * q + 1] = __float_as_uint(tv.y);
          }
      } else {
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int q = 0; q < 4; q++)
            r[8 * a + 2 * q] = __float_as_uint(acc[4 * h + a][q].x), r[8 * a + 2 * q + 1] = __float_as_uint(acc[4 * h + a][q].y);
      }
      tmem_st32(tcol + 32 * h, r);
    }
  }
  tmem_st_wait();
  __syncthreads();  // every stage consumed: the weight / raw region takes the whole y2 rows
  float* y2s = sm;
  for (int e = t; e < C3C_IN * (C3C_YROW / 4); e += C3C_THREADS) {
    const int ri = e / (C3C_YROW / 4), q = e - ri * (C3C_YROW / 4), g = r0 - 1 + ri;
    if (g >= 0 && g < total)
      cp_async16(y2s + ri * C3C_YROW + 4 * q, y2 + static_cast<int64_t>(g) * C3C_YROW + 4 * q);
    else
      *reinterpret_cast<float4*>(y2s + ri * C3C_YROW + 4 * q) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();
  {  // patch norms: warp w takes positions w, w+8, ...; lanes split the 576 taps
    const int lane = t & 31;
    for (int n = warp; n < C3C_N; n += C3C_THREADS / 32) {
      const int rho = n / 20, f = n - 20 * rho;
      float ss = 0.0f;
      for (int k = lane; k < K3; k += 32) {
        const int e = ko[k];
        const float a = valid[rho * 3 + (e >> 16)] ? y2s[rho * C3C_YROW + 2 * f + (e & 0xffff)] : 0.0f;
        ss = __fmaf_rn(a, a, ss);
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      // fp32 sum of 576 squares: relative error below 2^-14; inflate past it
      if (lane == 0) na[n] = __fmul_ru(__fsqrt_ru(ss), 1.0f + 0x1p-12f);
    }
  }
  __syncthreads();
  // y~ (relu of the totals) for half h of the thread's elements: a in [4h, 4h+4), all b
  auto load_y = [&](int h, float (&y)[4][8]) {
    uint32_t r[32];
    tmem_ld32(tcol + 32 * h, r);
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int b = 0; b < 8; b++) y[a][b] = fmaxf(__uint_as_float(r[8 * a + b]), 0.0f);
  };
  auto bound = [&](int a, int b) { return __fmul_ru(__fmul_ru(C3C_BOUND, na[c3c_n(pg, b)]), nw[c3c_o(cg, a)]); };
  {  // each row's lower bound of its maximum; positions 4pg.. lie in row pA, 40+4pg.. in row pB
    float loA = 0.0f, loB = 0.0f;
#pragma unroll
    for (int h = 0; h < 2; h++) {
      float y[4][8];
      load_y(h, y);
      if (act) {
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int b = 0; b < 4; b++) {
            loA = fmaxf(loA, __fsub_rd(y[a][b], bound(4 * h + a, b)));
            loB = fmaxf(loB, __fsub_rd(y[a][b + 4], bound(4 * h + a, b + 4)));
          }
      }
    }
    if (act && loA > 0.0f) atomicMax(reinterpret_cast<int*>(rowL + (4 * pg) / 20), __float_as_int(loA));
    if (act && loB > 0.0f) atomicMax(reinterpret_cast<int*>(rowL + (40 + 4 * pg) / 20), __float_as_int(loB));
  }
  __syncthreads();
  // candidates for each row's maximum -> the list (overflow: the whole block runs exactly)
  auto push = [&](int rho, int o, int f) {
    const int e = atomicAdd(cnt, 1);
    if (e < C3C_CAP) lst[e] = (rho << 16) | (o << 5) | f; else *ovf = 1;
  };
#pragma unroll
  for (int h = 0; h < 2; h++) {
    float y[4][8];
    load_y(h, y);
    if (act) {
#pragma unroll
      for (int a = 0; a < 4; a++)
#pragma unroll
        for (int b = 0; b < 8; b++) {
          const int n = c3c_n(pg, b), rho = n / 20;
          if (r0 + rho < total && __fadd_ru(y[a][b], bound(4 * h + a, b)) >= rowL[rho])
            push(rho, c3c_o(cg, 4 * h + a), n - 20 * rho);
        }
    }
  }
  __syncthreads();
  const int ncand = min(*cnt, C3C_CAP);
  const bool overflow = *ovf != 0;
  const int grp = t >> 3, l = t & 7;
  if (!overflow) {  // reference-order values of the candidates; each row's exact maximum
    for (int b0 = 0; b0 < ncand; b0 += C3C_THREADS / 8) {
      const int e = b0 + grp, en = lst[min(e, ncand - 1)];
      const float v = c3c_fold(c3c_lane(y2s, c3, ko, valid, en >> 16, (en >> 5) & 255, en & 31, l));
      if (e < ncand && l == 0) {
        lval[e] = v;
        atomicMax(reinterpret_cast<int*>(rowM + (en >> 16)), __float_as_int(v));
      }
    }
  }
  __syncthreads();
  if (t < C3C_R) rowInv[t] = quant_inv(quant_scale(rowM[t]));
  __syncthreads();
  if (overflow) {  // every element in reference order (rows whose bounds cannot separate anything)
    for (int b0 = 0; b0 < C3C_R * FLAT; b0 += C3C_THREADS / 8) {
      const int e = b0 + grp, rho = e / FLAT, rem = e - rho * FLAT, o = rem / 20, f = rem - 20 * o;
      const float v = c3c_fold(c3c_lane(y2s, c3, ko, valid, rho, o, f, l));
      if (l == 0 && r0 + rho < total) atomicMax(reinterpret_cast<int*>(rowM + rho), __float_as_int(v));
    }
    __syncthreads();
    for (int b0 = 0; b0 < C3C_R * FLAT; b0 += C3C_THREADS / 8) {
      const int e = b0 + grp, rho = e / FLAT, rem = e - rho * FLAT, o = rem / 20, f = rem - 20 * o;
      const float v = c3c_fold(c3c_lane(y2s, c3, ko, valid, rho, o, f, l));
      if (l == 0 && r0 + rho < total) qo[rho * FLAT + o * 20 + f] = quant_one(v, quant_inv(quant_scale(rowM[rho])));
    }
  } else {
    // every element that is neither a candidate nor near a rounding boundary is quantised from
    // y~; the rest join the list after the candidates
#pragma unroll
    for (int h = 0; h < 2; h++) {
      float y[4][8];
      load_y(h, y);
      if (act) {
#pragma unroll
        for (int a = 0; a < 4; a++)
#pragma unroll
          for (int b = 0; b < 8; b++) {
            const int n = c3c_n(pg, b), rho = n / 20, f = n - 20 * rho, o = c3c_o(cg, 4 * h + a);
            const float E = bound(4 * h + a, b);
            if (r0 + rho >= total || __fadd_ru(y[a][b], E) >= rowL[rho]) continue;
            const float inv = rowInv[rho];
            const float lim = __fsub_rd(0.5f, __fadd_ru(__fmul_ru(E, inv), 0x1p-16f));
            const float sv = __fmaf_rn(y[a][b], inv, RINT_MAGIC);
            const float d = __fmaf_rn(y[a][b], inv, __fsub_rn(RINT_MAGIC, sv));
            if (fabsf(d) < lim)
              qo[rho * FLAT + o * 20 + f] = static_cast<int8_t>(__float_as_uint(sv) & 0xffu);
            else
              push(rho, o, f);
          }
      }
    }
    __syncthreads();
    const int ntot = min(*cnt, C3C_CAP);
    if (*ovf) {  // the near-boundary list overflowed: its entries past the cap are not recorded
      for (int b0 = 0; b0 < C3C_R * FLAT; b0 += C3C_THREADS / 8) {
        const int e = b0 + grp, rho = e / FLAT, rem = e - rho * FLAT, o = rem / 20, f = rem - 20 * o;
        const float v = c3c_fold(c3c_lane(y2s, c3, ko, valid, rho, o, f, l));
        if (l == 0 && r0 + rho < total) qo[rho * FLAT + o * 20 + f] = quant_one(v, rowInv[rho]);
      }
    } else {
      for (int e = t; e < ncand; e += C3C_THREADS) {  // the candidates' values are known
        const int en = lst[e], rho = en >> 16;
        qo[rho * FLAT + ((en >> 5) & 255) * 20 + (en & 31)] = quant_one(lval[e], rowInv[rho]);
      }
      for (int b0 = ncand; b0 < ntot; b0 += C3C_THREADS / 8) {
        const int e = b0 + grp, en = lst[min(e, ntot - 1)], rho = en >> 16;
        const float v = c3c_fold(c3c_lane(y2s, c3, ko, valid, rho, (en >> 5) & 255, en & 31, l));
        if (e < ntot && l == 0) qo[rho * FLAT + ((en >> 5) & 255) * 20 + (en & 31)] = quant_one(v, rowInv[rho]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(*tslot, 128);
  }
  for (int rho = 0; rho < C3C_R; rho++) {
    const int r = r0 + rho;
    if (r >= total) break;
    const int4* src = reinterpret_cast<const int4*>(qo + rho * FLAT);
    int4* dst = reinterpret_cast<int4*>(xq + static_cast<int64_t>(r) * FLAT);
    for (int e = t; e < FLAT / 16; e += C3C_THREADS) dst[e] = src[e];
    if (t == 0) xs[r] = quant_scale(rowM[rho]);
  }
}

// c3t[k][o] = c3[o][k] (the stage tiles of conv3_cert_k) and nw[o] >= |c3[o] o n|_2, n(k) the
// rounding depth of tap k in the two summation orders (see the bound above), from the double
// sum of squares rounded up; once per model
__device__ __forceinline__ int c3c_depth(int k) {
  const int c = k / 8, l = k % 8, s = k / C3C_KS, i = k % C3C_KS;
  return 1 + (72 - c) + (l < 2 ? 7 : 8 - l) + (C3C_KS - i) + (s == 0 ? C3C_NST - 1 : C3C_NST - s);
}
__global__ void conv3_cert_prep_k(const float* __restrict__ c3, float* __restrict__ c3t, float* __restrict__ nw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < K3 * C3) {
    const int k = i / C3, o = i - k * C3;
    c3t[i] = c3[static_cast<int64_t>(o) * K3 + k];
  }
  if (i < C3) {
    double ss = 0.0;
    for (int k = 0; k < K3; k++) {
      const double w = static_cast<double>(c3[static_cast<int64_t>(i) * K3 + k]) * c3c_depth(k);
      ss += w * w;
    }
    nw[i] = __double2float_ru(__dsqrt_ru(ss) * (1.0 + 0x1p-40));
  }
}

// ------------------------------------------------------------------------ GELU + quant
// in place x = gelu(x) (src/model.rs:495,710-712), then per-row quant; one warp per row.
__global__ void __launch_bounds__(256) gelu_quant_k(float* __restrict__ x, int m, int k, int8_t* __restrict__ xq,
                                                    float* __restrict__ xs) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= m) return;
  float* r = x + static_cast<int64_t>(row) * k;
  float mx = 0.0f;
  for (int j = lane; j < k; j += 32) {
    const float v = gelu_ref(r[j]);
    r[j] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = warp_max(mx);
  const float sc = quant_scale(mx), inv = quant_inv(sc);
  for (int j = lane; j < k; j += 32) xq[static_cast<int64_t>(row) * k + j] = quant_one(r[j], inv);
  if (lane == 0) xs[row] = sc;
}

// GELU + per-row quant of a read-only [m][k] input (the FF1 GEMM output): the GELU values are
// only needed to quantise, so they are staged in shared memory (one warp per row, 8 rows per
// block) and never written back.  Same results as gelu in place followed by quant.
constexpr int GQ_ROWS = 4;

__global__ void __launch_bounds__(256) gelu_quant_ro_k(const float* __restrict__ y, int m, int k,
                                                       int8_t* __restrict__ xq, float* __restrict__ xs) {
  extern __shared__ float gsm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * GQ_ROWS + warp;
  if (row >= m) return;
  float* g = gsm + static_cast<size_t>(warp) * k;
  const float* r = y + static_cast<int64_t>(row) * k;
  int8_t* q = xq + static_cast<int64_t>(row) * k;
  float mx = 0.0f;
  if ((k & 255) == 0 && (reinterpret_cast<uintptr_t>(r) & 15) == 0) {
    // eight independent GELUs per lane per step (columns j .. j+3 and j+128 .. j+131): the long
    // exact tanh chains overlap; the next step's row values are loaded before this step's GELUs
    float4 nv0 = __ldg(reinterpret_cast<const float4*>(r + lane * 4));
    float4 nv1 = __ldg(reinterpret_cast<const float4*>(r + lane * 4 + 128));
#pragma unroll 1
    for (int j = lane * 4; j < k; j += 256) {
      const float4 v0 = nv0, v1 = nv1;
      if (j + 256 < k) {
        nv0 = __ldg(reinterpret_cast<const float4*>(r + j + 256));
        nv1 = __ldg(reinterpret_cast<const float4*>(r + j + 384));
      }
      const float2 ga = gelu_ref2(make_float2(v0.x, v0.y)), gb = gelu_ref2(make_float2(v0.z, v0.w));
      const float2 gc = gelu_ref2(make_float2(v1.x, v1.y)), gd = gelu_ref2(make_float2(v1.z, v1.w));
      const float4 g0 = make_float4(ga.x, ga.y, gb.x, gb.y), g1 = make_float4(gc.x, gc.y, gd.x, gd.y);
      *reinterpret_cast<float4*>(g + j) = g0;
      *reinterpret_cast<float4*>(g + j + 128) = g1;
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(g0.x), fabsf(g0.y)), fmaxf(fabsf(g0.z), fabsf(g0.w))));
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(g1.x), fabsf(g1.y)), fmaxf(fabsf(g1.z), fabsf(g1.w))));
    }
    mx = warp_max(mx);
    const float sc = quant_scale(mx), inv = quant_inv(sc);
    for (int j = lane * 4; j < k; j += 128) {
      const float4 gv = *reinterpret_cast<const float4*>(g + j);
      char4 c;
      c.x = quant_one(gv.x, inv); c.y = quant_one(gv.y, inv); c.z = quant_one(gv.z, inv); c.w = quant_one(gv.w, inv);
      *reinterpret_cast<char4*>(q + j) = c;
    }
    if (lane == 0) xs[row] = sc;
    return;
  }
#pragma unroll 1
  for (int j = lane; j < k; j += 32) {
    const float v = gelu_ref(__ldg(r + j));
    g[j] = v;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = warp_max(mx);
  const float sc = quant_scale(mx), inv = quant_inv(sc);
  for (int j = lane; j < k; j += 32) q[j] = quant_one(g[j], inv);
  if (lane == 0) xs[row] = sc;
}

// One row of GELU + quant done exactly by warp `lane`s (two passes of gelu_ref over the
// row): the certified kernel's path for rows holding a non-finite approximate value.
__device__ __noinline__ void gelu_quant_row_exact(const float* __restrict__ r, int k, int lane, int8_t* __restrict__ q,
                                                  float* __restrict__ xs) {
  float mx = 0.0f;
  for (int j = lane; j < k; j += 32) mx = fmaxf(mx, fabsf(gelu_ref(r[j])));
  mx = warp_max(mx);
  const float sc = quant_scale(mx), inv = quant_inv(sc);
  for (int j = lane; j < k; j += 32) q[j] = quant_one(gelu_ref(r[j]), inv);
  if (lane == 0) *xs = sc;
}

// GELU + per-row quant with the certified approximation (gelu_fast2, common.cuh): one warp per
// row of k = 128 NV columns, lane l holding columns 4l + 128i + c in registers.
//  1. g~ = gelu_fast(x) for the row, and max x.
//  2. The exact maximum M = max |g|: gelu_ref is non-decreasing on [0, inf] and |gelu_ref| <=
//     GELU_NEG_MAX below 0 (both checked on every float), so M = gelu_ref(max x) whenever that is
//     >= GELU_NEG_MAX.  Otherwise (rows of small or negative values) M is attained at an element
//     with |g~| >= mt - 2E, mt = max |g~|, E = A + B mt (it has |g| >= |g~_a| - E = mt - E for
//     the approximate argmax a, so |g~| >= mt - 2E; every other element has |g| < mt - E <= M),
//     and is the maximum of gelu_ref over those candidates.  sc, inv follow from M as in quant,
//     and every |g~ - g| <= E = A + B (M + A)(1 + 2B), since |g~| <= (M + A) / (1 - B).
//  3. With w = g~ * inv (exact real product), the exact v = RN(g * inv) lies within
//     E inv + 2^-18 of w (half an ulp of values below 128).  s = fma(g~, inv, 1.5 * 2^23) rounds
//     w to the nearest integer n (ties to even), held in the low mantissa bits of s for
//     |w| < 2^22; n = s - 1.5 * 2^23 exactly, and d = fma(g~, inv, -n) is w - n within 2^-25.
//     If |d| < lim = 1/2 - (E inv + 2^-16), then |v - n| < 1/2: round(v) = n, and |v| <= 127
//     needs no clamp; the low byte of s's bits is n as an int8, without conversions.  The other
//     elements (rare; every element of a row whose bound reaches 1/2, and NaN distances) are
//     quantised again from gelu_ref.
// The int8 row and its scale are therefore identical to quant(gelu(x)) on every input.
// Persistent warps: each takes rows w, w + W, ...; while it works on one row, the next streams
// into the other half of its two-row shared-memory buffer by cp.async (each lane copies and
// later reads only its own 16-byte pieces, so no synchronisation beyond the copy wait).
constexpr int GQ_WARPS = 4;              // warps per block
template <int NV>
__global__ void __launch_bounds__(32 * GQ_WARPS, 3) gelu_quant_cert_k(const float* __restrict__ y, int m,
                                                                      int8_t* __restrict__ xq,
                                                                      float* __restrict__ xs) {
  static_assert(NV >= 1 && NV <= 16, "a lane's candidate mask holds 64 elements");
  constexpr int K = 128 * NV;
  extern __shared__ __align__(16) float gq_sm[];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5, nwarps = gridDim.x * GQ_WARPS;
  float* buf = gq_sm + wib * 2 * K + 4 * lane;  // [2][K] per warp, this lane's columns
  int row = blockIdx.x * GQ_WARPS + wib;
  if (row < m) {
#pragma unroll
    for (int i = 0; i < NV; i++) cp_async16(buf + 128 * i, y + static_cast<int64_t>(row) * K + 4 * lane + 128 * i);
  }
  cp_async_commit();
  for (int it = 0; row < m; row += nwarps, it ^= 1) {
    cp_async_wait<0>();
    if (row + nwarps < m) {
#pragma unroll
      for (int i = 0; i < NV; i++)
        cp_async16(buf + (it ^ 1) * K + 128 * i, y + static_cast<int64_t>(row + nwarps) * K + 4 * lane + 128 * i);
    }
    cp_async_commit();
    const float* r = y + static_cast<int64_t>(row) * K + 4 * lane;
    int8_t* q = xq + static_cast<int64_t>(row) * K + 4 * lane;
    float g[NV][4];
    float xm = -3.40282347e+38f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const float4 v = *reinterpret_cast<const float4*>(buf + it * K + 128 * i);
      g[i][0] = v.x, g[i][1] = v.y, g[i][2] = v.z, g[i][3] = v.w;
      xm = fmaxf(fmaxf(xm, fmaxf(v.x, v.y)), fmaxf(v.z, v.w));
    }
    float2 chk = make_float2(0.0f, 0.0f);  // stays 0 unless some g~ is inf or NaN (inf * 0 = NaN)
#pragma unroll
    for (int i = 0; i < NV; i++)
#pragma unroll
      for (int c = 0; c < 4; c += 2) {
        const float2 v = gelu_fast2(make_float2(g[i][c], g[i][c + 1]));
        g[i][c] = v.x, g[i][c + 1] = v.y;
        chk = fma2_rn(v, f2c(0.0f), chk);
      }
    if (__any_sync(0xffffffffu, !(chk.x == 0.0f) || !(chk.y == 0.0f))) {
      gelu_quant_row_exact(y + static_cast<int64_t>(row) * K, K, lane, xq + static_cast<int64_t>(row) * K, xs + row);
      continue;
    }
    float mx = gelu_ref(warp_max(xm));
    if (!(mx >= GELU_NEG_MAX)) {  // the maximum from the exact GELU of the candidates
      float mt = 0.0f;
#pragma unroll
      for (int i = 0; i < NV; i++)
#pragma unroll
        for (int c = 0; c < 4; c++) mt = fmaxf(mt, fabsf(g[i][c]));
      const float lane_mt = mt;
      mt = warp_max(mt);
      const float L = __fsub_rd(mt, __fmul_ru(2.0f, __fmaf_ru(GELU_CERT_B, mt, GELU_CERT_A)));
      mx = 0.0f;
      if (lane_mt >= L) {  // this lane holds candidates
        unsigned long long cand = 0;
#pragma unroll
        for (int i = 0; i < NV; i++)
#pragma unroll
          for (int c = 0; c < 4; c++) cand |= static_cast<unsigned long long>(fabsf(g[i][c]) >= L) << (4 * i + c);
        while (cand) {
          const int b = __ffsll(static_cast<long long>(cand)) - 1;
          cand &= cand - 1;
          mx = fmaxf(mx, fabsf(gelu_ref(r[128 * (b >> 2) + (b & 3)])));
        }
      }
      mx = warp_max(mx);
    }
    const float E = __fmaf_ru(GELU_CERT_B, __fmul_ru(__fadd_ru(mx, GELU_CERT_A), 1.0f + 2.0f * GELU_CERT_B), GELU_CERT_A);
    const float sc = quant_scale(mx), inv = quant_inv(sc);
    const float lim = __fsub_rd(0.5f, __fadd_ru(__fmul_ru(E, inv), 0x1p-16f));
    bool amb = false;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      uint32_t b[4];
#pragma unroll
      for (int c = 0; c < 4; c += 2) {
        const float2 gg = make_float2(g[i][c], g[i][c + 1]);
        const float2 sv = fma2_rn(gg, f2c(inv), f2c(RINT_MAGIC));
        const float2 d = fma2_rn(gg, f2c(inv), psub2(f2c(RINT_MAGIC), sv));
        amb |= !(fabsf(d.x) < lim) || !(fabsf(d.y) < lim);
        b[c] = __float_as_uint(sv.x), b[c + 1] = __float_as_uint(sv.y);
      }
      *reinterpret_cast<uint32_t*>(q + 128 * i) =
          __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
    }
    if (lane == 0) xs[row] = sc;
    if (amb) {  // quantise the elements near a rounding boundary again from the exact GELU
      unsigned long long mask = 0;
#pragma unroll
      for (int i = 0; i < NV; i++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const float d = __fmaf_rn(g[i][c], inv, __fsub_rn(RINT_MAGIC, __fmaf_rn(g[i][c], inv, RINT_MAGIC)));
          mask |= static_cast<unsigned long long>(!(fabsf(d) < lim)) << (4 * i + c);
        }
      while (mask) {
        const int b = __ffsll(static_cast<long long>(mask)) - 1;
        mask &= mask - 1;
        const int col = 128 * (b >> 2) + (b & 3);
        q[col] = quant_one(gelu_ref(r[col]), inv);
      }
    }
  }
}

// Exhaustive check of the facts gelu_quant_cert_k relies on, over the float bit patterns
// [start, start + count) (both even), into stats[8]:
//   [0] max over inputs with both values finite of |g~ - g| - GELU_CERT_B |g~| (a non-negative
//       double's bits), [1] inputs where gelu_ref is non-finite and gelu_fast finite, [2] inputs
//       with both finite and |g~ - g| > GELU_CERT_A + GELU_CERT_B |g~|, [3] inputs where only
//       gelu_fast is non-finite (allowed: such rows run exactly), [4] max |g~ - g| / |g~| over
//       |g~| >= 2^-4 and [5] max |g~ - g| over |g~| < 2^-4 (double bits, for choosing A and B),
//   [6] pairs of adjacent floats 0 <= x < x' <= inf with gelu_ref(x') < gelu_ref(x), [7] max of
//       |gelu_ref(x)| over non-NaN x < 0 (double bits).
__global__ void gelu_cert_scan_k(unsigned long long start, unsigned long long count,
                                 unsigned long long* __restrict__ stats) {
  double worst = 0.0, rel_max = 0.0, abs_small = 0.0, neg_max = 0.0;
  unsigned long long n_nf = 0, n_viol = 0, n_fast_nf = 0, n_mono = 0;
  const unsigned long long stride = 2ull * gridDim.x * blockDim.x;
  for (unsigned long long i = 2ull * (blockIdx.x * blockDim.x + threadIdx.x); i < count; i += stride) {
    const uint32_t b0 = static_cast<uint32_t>(start + i);
    const float x[2] = {__uint_as_float(b0), __uint_as_float(b0 + 1)};
    const float2 gf = gelu_fast2(make_float2(x[0], x[1]));
    const float gx[2] = {gelu_ref(x[0]), gelu_ref(x[1])}, fx[2] = {gf.x, gf.y};
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const bool fin_r = fabsf(gx[u]) <= 3.40282347e+38f, fin_f = fabsf(fx[u]) <= 3.40282347e+38f;
      if (!fin_r && fin_f) n_nf++;
      if (fin_r && !fin_f) n_fast_nf++;
      if (fin_r && fin_f) {
        const double err = fabs(static_cast<double>(fx[u]) - static_cast<double>(gx[u]));
        const double af = fabs(static_cast<double>(fx[u]));
        const double rel = static_cast<double>(GELU_CERT_B) * af;
        worst = fmax(worst, err - rel);
        if (err > static_cast<double>(GELU_CERT_A) + rel) n_viol++;
        if (af >= 0x1p-4) rel_max = fmax(rel_max, err / af);
        else abs_small = fmax(abs_small, err);
      }
      const uint32_t bu = b0 + u;
      if (bu > 0x80000000u && bu <= 0xff800000u) neg_max = fmax(neg_max, fabs(static_cast<double>(gx[u])));
    }
    if (b0 < 0x7f800000u) {  // x0 < x1 <= inf, and x1 < x2 when x1 is finite
      if (gx[1] < gx[0]) n_mono++;
      if (b0 + 1 < 0x7f800000u && gelu_ref(__uint_as_float(b0 + 2)) < gx[1]) n_mono++;
    }
  }
  atomicMax(stats, static_cast<unsigned long long>(__double_as_longlong(worst)));
  if (n_nf) atomicAdd(stats + 1, n_nf);
  if (n_viol) atomicAdd(stats + 2, n_viol);
  if (n_fast_nf) atomicAdd(stats + 3, n_fast_nf);
  atomicMax(stats + 4, static_cast<unsigned long long>(__double_as_longlong(rel_max)));
  atomicMax(stats + 5, static_cast<unsigned long long>(__double_as_longlong(abs_small)));
  if (n_mono) atomicAdd(stats + 6, n_mono);
  atomicMax(stats + 7, static_cast<unsigned long long>(__double_as_longlong(neg_max)));
}

__global__ void add_k(float* __restrict__ h, const float* __restrict__ a, size_t n) {
  const size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n && ((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(a)) & 15) == 0) {
    float4 x = *reinterpret_cast<float4*>(h + i);
    const float4 y = *reinterpret_cast<const float4*>(a + i);
    *reinterpret_cast<float4*>(h + i) =
        make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z), __fadd_rn(x.w, y.w));
  } else {
    for (size_t j = i; j < i + 4 && j < n; j++) h[j] = __fadd_rn(h[j], a[j]);
  }
}

// row argmax, first maximum wins (src/model.rs:499-500): one block per row.
__global__ void __launch_bounds__(256) argmax_k(const float* __restrict__ x, int n, uint32_t* __restrict__ out) {
  __shared__ float bv[256];
  __shared__ int bi[256];
  const float* r = x + static_cast<int64_t>(blockIdx.x) * n;
  float best = -3.40282347e+38f;
  int bj = 0x7FFFFFFF;
  for (int j = threadIdx.x; j < n; j += blockDim.x)
    if (r[j] > best) { best = r[j]; bj = j; }
  bv[threadIdx.x] = best;
  bi[threadIdx.x] = bj;
  __syncthreads();
  for (int st = blockDim.x / 2; st > 0; st >>= 1) {
    if (threadIdx.x < st) {
      const float v2 = bv[threadIdx.x + st];
      const int i2 = bi[threadIdx.x + st];
      if (v2 > bv[threadIdx.x] || (v2 == bv[threadIdx.x] && i2 < bi[threadIdx.x])) {
        bv[threadIdx.x] = v2;
        bi[threadIdx.x] = i2;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = bi[0] == 0x7FFFFFFF ? 0u : static_cast<uint32_t>(bi[0]);
}

__global__ void keys_to_ids_k(const unsigned long long* __restrict__ keys, int m, uint32_t* __restrict__ ids) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= m) return;
  const unsigned long long k = keys[i];
  ids[i] = k == 0ull ? 0u : 0xFFFFFFFFu - static_cast<uint32_t>(k & 0xFFFFFFFFull);
}

// ------------------------------------------------------------------------ attention
// One block per (query tile, head).  A segment of t rows is cut into ceil(t/64) tiles of
// equal size (at most 64 rows), so short last tiles do not waste work; `tord` (optional)
// lists the tiles longest segment first, so the longest blocks start in the first wave.
// Scores s_ij = dotf(q_i, k_j) * 0.125 (src/kernels.rs:172-183 order); softmax
// e_j = exp(s_j - max), z = sequential sum, p_j = e_j / z; o_i[d] = sum over j in order of
// p_j * v_j[d] from 0 (src/model.rs:714-738).  Every element keeps the reference's exact
// sequence of rounded multiplies and adds.
//
// Register tiles.  Scores: lane p of every warp owns the tile's row pair (2p, 2p+1), and warp w
// a contiguous run of 4-key chunks; a thread holds its row pair x 4 keys with all 8 dotf lanes of
// each score as 4 float2 (lane l holds dims 8c + l), so the lane fold is 7 adds in one thread,
// in the reference order.  A lane's first step starts from the product itself rather than
// 0 + product: the two differ at most in the sign of a zero, which no later step can see (a
// zero score enters the softmax only through s - max and exp).  Each warp streams its chunks
// through a private double buffer (cp.async, warp-level sync only); Q is staged once with its
// 16-byte chunks XOR-swizzled by row pair.  PV: a thread owns row pairs (2p, 2p+1) for
// p = pa, pa+1 x head dims d0..d0+3; the accumulators pair (row 2p, dim d) with (row 2p+1,
// dim d^1); V chunks of 32 keys stream through two shared buffers, one barrier per chunk.
// Shared layout: exp table | Q [64][64] + key chunks [8 warps][2][4][64] + per-warp maxima
// [8][64] (scores) / V [2][32][64] (PV) | S2 [32 row pairs][sp] float2 | ZY [32][4] | Mx [64].
// Softmax: the row maxima are the maxima of the warps' running maxima; the exp and divide
// passes run flat over (row pair, key) with every thread on independent elements; z is one
// thread per row.
constexpr int ATT_KC = 32;   // keys per chunk
constexpr int ATT_RS = 68;   // row stride in floats that sizes the Q/K/V region
constexpr int ATT_A = (ATT_QT + 2 * ATT_KC) * ATT_RS;  // floats of the Q/K (and V) region
static_assert(2 * ATT_QT * HD + 8 * ATT_QT <= ATT_A, "score phase: Q, the warps' key chunks and maxima");
static_assert(2 * ATT_KC * HD <= ATT_A, "PV phase: two V chunks");

__host__ __device__ inline int att_pair_stride(int max_t1) { return ((max_t1 + 15) / 16) * 16 + 1; }

size_t attention_smem_bytes(int max_t1) {
  const int sp = att_pair_stride(max_t1);
  return 32 * 8 + static_cast<size_t>(ATT_A) * 4 + static_cast<size_t>(ATT_QT / 2) * sp * 8 + 3 * ATT_QT * 4;
}

__device__ __forceinline__ float2 lo2(float4 a) { return make_float2(a.x, a.y); }
__device__ __forceinline__ float2 hi2(float4 a) { return make_float2(a.z, a.w); }

// rows [j0, j0+nj) of K / V / Q for head h into dst (row stride ds floats); rows past nj are
// left as they are (never used).  16-byte copies when the source rows allow them.
__device__ __forceinline__ void att_copy_rows(float* dst, int ds, const float* __restrict__ src, int ld, int r0,
                                              int nj, int h, int tid, bool a16) {
  for (int e = tid; e < nj * 16; e += 256) {
    const int j = e >> 4, d4 = (e & 15) * 4;
    const float* g = src + static_cast<int64_t>(r0 + j) * ld + h * HD + d4;
    float* d = dst + j * ds + d4;
    if (a16) {
      cp_async16(d, g);
    } else {
#pragma unroll
      for (int u = 0; u < 4; u++) cp_async4(d + u, g + u);
    }
  }
  cp_async_commit();
}

// Scores of one 4-key chunk (NK valid keys, rows kept 64 floats apart at Kc) for the row pair
// (2p, 2p+1) of the swizzled Q tile (16-byte chunk d4 of row r at d4 ^ ((r >> 1) & 7)): all 8
// dotf lanes of each score in this thread, folded in lane order; score pairs to outp[u]; mx
// keeps the running maxima of the rows that exist (live0 / live1).
template <int NK>
__device__ __forceinline__ void att_score4(const float* Qs, int p, const float* Kc, float2* outp, float (&mx)[2],
                                           bool live0, bool live1) {
  const float* Q0 = Qs + 2 * p * HD;
  const int sw = p & 7;
  float2 acc[2][NK][4];
#pragma unroll
  for (int c = 0; c < 8; c++) {
    float4 qv[2][2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      qv[r][0] = *reinterpret_cast<const float4*>(Q0 + r * HD + 4 * ((2 * c) ^ sw));
      qv[r][1] = *reinterpret_cast<const float4*>(Q0 + r * HD + 4 * ((2 * c + 1) ^ sw));
    }
#pragma unroll
    for (int u = 0; u < NK; u++) {
      const float4 k0 = *reinterpret_cast<const float4*>(Kc + u * HD + 8 * c);
      const float4 k1 = *reinterpret_cast<const float4*>(Kc + u * HD + 8 * c + 4);
#pragma unroll
      for (int r = 0; r < 2; r++) {
        const float2 p0 = mulp(lo2(qv[r][0]), lo2(k0)), p1 = mulp(hi2(qv[r][0]), hi2(k0));
        const float2 p2 = mulp(lo2(qv[r][1]), lo2(k1)), p3 = mulp(hi2(qv[r][1]), hi2(k1));
        if (c == 0) {
          acc[r][u][0] = p0, acc[r][u][1] = p1, acc[r][u][2] = p2, acc[r][u][3] = p3;
        } else {
          acc[r][u][0] = add2_rn(acc[r][u][0], p0);
          acc[r][u][1] = add2_rn(acc[r][u][1], p1);
          acc[r][u][2] = add2_rn(acc[r][u][2], p2);
          acc[r][u][3] = add2_rn(acc[r][u][3], p3);
        }
      }
    }
  }
#pragma unroll
  for (int u = 0; u < NK; u++) {
    float sc[2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
      float x = __fadd_rn(acc[r][u][0].x, acc[r][u][0].y);
#pragma unroll
      for (int l = 1; l < 4; l++) x = __fadd_rn(__fadd_rn(x, acc[r][u][l].x), acc[r][u][l].y);
      sc[r] = __fmul_rn(x, 0.125f);
    }
    outp[u] = make_float2(sc[0], sc[1]);
    if (live0) mx[0] = fmaxf(mx[0], sc[0]);
    if (live1) mx[1] = fmaxf(mx[1], sc[1]);
  }
}

// Softmax passes over the flat element list e = p * t + j of a tile's row pairs p (float2
// per key j): element e of batch slot k is e0 + 256k.  Loads are clamped to the last element
// and every exp / quotient is computed unconditionally, so the NB pairs of a batch overlap;
// only the stores are guarded.  (e + 0.5) / t in float recovers p exactly for p < 32 and
// t < 2^16: its error is below 32 * 2^-23 = 2^-18 while its distance to an integer is at least
// 1 / (2t) > 2^-17.
__device__ __forceinline__ int att_pair(int e, float inv_t) {
  return static_cast<int>(__fmul_rn(__fadd_rn(static_cast<float>(e), 0.5f), inv_t));
}
template <int NB>
__device__ __forceinline__ void att_exp_batch(float2* S2, const float2* M2, const unsigned long long* tab, int sp, int t,
                                              float inv_t, int E, int e0) {
  float2 a[NB], m[NB];
  int off[NB];
#pragma unroll
  for (int k = 0; k < NB; k++) {
    const int e = min(e0 + 256 * k, E - 1), p = att_pair(e, inv_t);
    off[k] = p * sp + (e - p * t);
    m[k] = M2[p];
    a[k] = S2[off[k]];
  }
#pragma unroll
  for (int k = 0; k < NB; k++)
    a[k] = make_float2(expf_ref_smem(__fsub_rn(a[k].x, m[k].x), tab), expf_ref_smem(__fsub_rn(a[k].y, m[k].y), tab));
#pragma unroll
  for (int k = 0; k < NB; k++)
    if (e0 + 256 * k < E) S2[off[k]] = a[k];
}
// p = e / z with zy[p] = (z_2p, z_2p+1, rcp z_2p, rcp z_2p+1)
template <int NB>
__device__ __forceinline__ void att_div_batch(float2* S2, const float4* ZY, int sp, int t, float inv_t, int E, int e0) {
  float2 a[NB], q[NB];
  float4 zy[NB];
  int off[NB];
  bool tiny = false;
#pragma unroll
  for (int k = 0; k < NB; k++) {
    const int e = min(e0 + 256 * k, E - 1), p = att_pair(e, inv_t);
    off[k] = p * sp + (e - p * t);
    zy[k] = ZY[p];
    a[k] = S2[off[k]];
  }
#pragma unroll
  for (int k = 0; k < NB; k++) {
    q[k] = make_float2(div_unit_fast(a[k].x, zy[k].x, zy[k].z), div_unit_fast(a[k].y, zy[k].y, zy[k].w));
    tiny |= div_unit_tiny(a[k].x) | div_unit_tiny(a[k].y);
  }
  if (__any_sync(0xffffffffu, tiny))  // numerators below 2^-80: the full division
#pragma unroll
    for (int k = 0; k < NB; k++) {
      if (div_unit_tiny(a[k].x)) q[k].x = __fdiv_rn(a[k].x, zy[k].x);
      if (div_unit_tiny(a[k].y)) q[k].y = __fdiv_rn(a[k].y, zy[k].y);
    }
#pragma unroll
  for (int k = 0; k < NB; k++)
    if (e0 + 256 * k < E) S2[off[k]] = q[k];
}
// runs batches of 4 slots, then the remainder (Kw slots in all for this warp)
#define ATT_BATCHES(FN, ...)                                   \
  {                                                            \
    int k0 = 0;                                                \
    for (; k0 + 4 <= Kw; k0 += 4) FN<4>(__VA_ARGS__, tid + 256 * k0); \
    switch (Kw - k0) {                                         \
      case 3: FN<3>(__VA_ARGS__, tid + 256 * k0); break;       \
      case 2: FN<2>(__VA_ARGS__, tid + 256 * k0); break;       \
      case 1: FN<1>(__VA_ARGS__, tid + 256 * k0); break;       \
      default: break;                                          \
    }                                                          \
  }

__global__ void __launch_bounds__(256, 2) attn_k(const float* __restrict__ q, const float* __restrict__ k,
                                                 const float* __restrict__ v, int ld, Segs s,
                                                 const int* __restrict__ toff, const int* __restrict__ tord,
                                                 int max_t1, float* __restrict__ out, int ldo) {
  extern __shared__ __align__(16) float sm[];
  const int sp = att_pair_stride(max_t1);
  unsigned long long* tab = reinterpret_cast<unsigned long long*>(sm);
  float* Q = sm + 64;                     // score phase: Q [64][64] | K chunks [8 warps][2][4][64] | maxima [8][64]
  float* Vb = Q;                          // [2][32][64] (PV phase)
  float2* S2 = reinterpret_cast<float2*>(Q + ATT_A);  // [32][sp]
  float* ZY = reinterpret_cast<float*>(S2 + (ATT_QT / 2) * sp);  // [32][4]: z and 1/z of each row pair
  float* Mx = ZY + 2 * ATT_QT;            // [64]: row maxima
  const int tile = tord ? tord[blockIdx.x] : blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  int sw = 0;
  if (toff) {
    int lo = 0, hi = s.n - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (toff[mid] <= tile) lo = mid; else hi = mid - 1;
    }
    sw = lo;
  }
  const int qt = toff ? tile - toff[sw] : tile;
  const int rb = s.row_begin(sw), t = s.rows(sw);
  const int ntile = (t + ATT_QT - 1) / ATT_QT, rpt = ntile > 0 ? (t + ntile - 1) / ntile : 0;
  const int i0 = qt * rpt;
  const int ni = min(rpt, t - i0);
  if (ni <= 0 || t > max_t1) return;
  const bool a16 = ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) &
                    15) == 0 &&
                   (ld & 3) == 0;
  if (tid < 32) tab[tid] = kExp2Tab[tid];
  const int warp = tid >> 5, lane = tid & 31;
  const int nchunks = (t + ATT_KC - 1) / ATT_KC;  // 32-key chunks of the PV loop
  // ---- scores.  The tile's rows go to the lanes (lane p: rows 2p, 2p+1), its keys to the warps
  // (warp w: 4-key chunks [w nc / 8, (w+1) nc / 8) of the nc = ceil(t / 4)), each warp streaming
  // its own chunks by cp.async into a private double buffer, so the loop needs no block barrier.
  // Q rows lie 64 floats apart with the 16-byte chunk d4 of row r at d4 ^ ((r >> 1) & 7): the 8
  // row pairs of a quarter warp hit 8 distinct bank groups, and the key loads are broadcasts.
  {
    float* Qs = Q;                                          // [64][64], swizzled
    float* Kw = Qs + ATT_QT * HD + warp * (2 * 4 * HD);     // [2][4][64] this warp's chunks
    float* Mw = Qs + 2 * ATT_QT * HD;                       // [8 warps][64 rows] maxima
    for (int e = tid; e < ni * 16; e += 256) {
      const int r = e >> 4, d4 = e & 15;
      const float* g = q + static_cast<int64_t>(rb + i0 + r) * ld + h * HD + 4 * d4;
      float* d = Qs + r * HD + 4 * (d4 ^ ((r >> 1) & 7));
      if (a16) {
        cp_async16(d, g);
      } else {
#pragma unroll
        for (int u = 0; u < 4; u++) cp_async4(d + u, g + u);
      }
    }
    cp_async_commit();
    const int nc = (t + 3) >> 2, cb = (warp * nc) >> 3, ce = ((warp + 1) * nc) >> 3;
    auto copy_chunk = [&](int c, int buf) {  // keys 4c .. 4c+3 (those below t)
      const int j0 = 4 * c, nk = min(4, t - j0);
      for (int e = lane; e < nk * 16; e += 32) {
        const int u = e >> 4, d4 = e & 15;
        const float* g = k + static_cast<int64_t>(rb + j0 + u) * ld + h * HD + 4 * d4;
        float* d = Kw + buf * 4 * HD + u * HD + 4 * d4;
        if (a16) {
          cp_async16(d, g);
        } else {
#pragma unroll
          for (int w4 = 0; w4 < 4; w4++) cp_async4(d + w4, g + w4);
        }
      }
      cp_async_commit();
    };
    if (cb < ce) copy_chunk(cb, 0);
    cp_async_wait<0>();
    __syncthreads();  // Q visible to every warp
    const bool live0 = 2 * lane < ni, live1 = 2 * lane + 1 < ni;
    float2* outp = S2 + lane * sp;
    float mx[2] = {-3.40282347e+38f, -3.40282347e+38f};
    for (int c = cb; c < ce; c++) {
      const int buf = (c - cb) & 1;
      if (c + 1 < ce) {
        copy_chunk(c + 1, buf ^ 1);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();  // chunk c landed for every lane of the warp
      const int j0 = 4 * c;
      const float* Kc = Kw + buf * 4 * HD;
      switch (min(4, t - j0)) {
        case 4: att_score4<4>(Qs, lane, Kc, outp + j0, mx, live0, live1); break;
        case 3: att_score4<3>(Qs, lane, Kc, outp + j0, mx, live0, live1); break;
        case 2: att_score4<2>(Qs, lane, Kc, outp + j0, mx, live0, live1); break;
        default: att_score4<1>(Qs, lane, Kc, outp + j0, mx, live0, live1); break;
      }
      __syncwarp();  // every lane is done with buffer buf before chunk c+2 goes into it
    }
    Mw[warp * ATT_QT + 2 * lane] = mx[0];
    Mw[warp * ATT_QT + 2 * lane + 1] = mx[1];
    __syncthreads();
    if (tid < ATT_QT) {
      float m = Mw[tid];
#pragma unroll
      for (int w = 1; w < 8; w++) m = fmaxf(m, Mw[w * ATT_QT + tid]);
      Mx[tid] = m;
    }
  }
  __syncthreads();  // scores and row maxima complete; the Q/K region is free
  // the first V chunk streams in while the softmax runs
  att_copy_rows(Vb, HD, v, ld, rb, min(ATT_KC, t), h, tid, a16);
  // ---- softmax: e = exp(s - max) flat over the npair * t row-pair elements; z per row (a
  // left fold, one thread per row) with its reciprocal; p = e / z flat again.  Kw: the slots of
  // this warp's first lane (later lanes clamp the one element they may lack)
  const int npair = (ni + 1) >> 1, E = npair * t, Kw = max(0, (E - warp * 32 + 255) >> 8);
  const float inv_t = 1.0f / static_cast<float>(t);
  ATT_BATCHES(att_exp_batch, S2, reinterpret_cast<const float2*>(Mx), tab, sp, t, inv_t, E)
  __syncthreads();
  float* Sf = reinterpret_cast<float*>(S2);
  if (tid < ni) {  // z: a left fold over j; the next 8 loads are issued before the current adds
    const float* row = Sf + (tid >> 1) * sp * 2 + (tid & 1);
    float z = 0.0f;
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; u++) x[u] = row[2 * min(u, t - 1)];
    int j = 0;
    for (; j + 8 <= t; j += 8) {
      float nx[8];
#pragma unroll
      for (int u = 0; u < 8; u++) nx[u] = row[2 * min(j + 8 + u, t - 1)];
#pragma unroll
      for (int u = 0; u < 8; u++) z = __fadd_rn(z, x[u]);
#pragma unroll
      for (int u = 0; u < 8; u++) x[u] = nx[u];
    }
#pragma unroll
    for (int u = 0; u < 7; u++)
      if (j + u < t) z = __fadd_rn(z, x[u]);
    ZY[4 * (tid >> 1) + (tid & 1)] = z;
    ZY[4 * (tid >> 1) + 2 + (tid & 1)] = __frcp_rn(z);
  } else if (tid == ni && (ni & 1)) {  // the unused second row of an odd tile's last pair
    ZY[4 * (tid >> 1) + 1] = 1.0f;
    ZY[4 * (tid >> 1) + 3] = 1.0f;
  }
  __syncthreads();
  ATT_BATCHES(att_div_batch, S2, reinterpret_cast<const float4*>(ZY), sp, t, inv_t, E)
  // ---- PV: warp w owns rows 8w .. 8w+7 (row pairs pa = 4w + 2rg and pa + 1 for lane half
  // rg) x dims 4dg .. 4dg+3 (dg = lane & 15): 4 rows x 4 dims per lane
  const int rg = lane >> 4, dg = lane & 15, pa = 4 * warp + 2 * rg;
  const bool live = 8 * warp < ni;  // warp-uniform
  float2 o[2][4];
#pragma unroll
  for (int a = 0; a < 2; a++)
#pragma unroll
    for (int u = 0; u < 4; u++) o[a][u] = make_float2(0.0f, 0.0f);
  for (int ch = 0; ch < nchunks; ch++) {
    const int j0 = ch * ATT_KC, nj = min(ATT_KC, t - j0);
    cp_async_wait<0>();
    __syncthreads();  // V chunk ch and all probabilities visible; chunk ch-1 consumed
    if (ch + 1 < nchunks)
      att_copy_rows(Vb + ((ch + 1) & 1) * ATT_KC * HD, HD, v, ld, rb + j0 + ATT_KC, min(ATT_KC, t - j0 - ATT_KC), h,
                    tid, a16);
    const float2* p0 = S2 + pa * sp + j0;
    const float2* p1 = p0 + sp;
    const float* vr = Vb + (ch & 1) * ATT_KC * HD + 4 * dg;
    if (live) {
#pragma unroll 8
      for (int jj = 0; jj < nj; jj++) {
        const float2 pa2 = p0[jj], pb2 = p1[jj];
        const float4 x = *reinterpret_cast<const float4*>(vr + jj * HD);
        o[0][0] = add2_rn(o[0][0], mulp(pa2, lo2(x)));
        o[0][1] = add2_rn(o[0][1], mulp(pa2, make_float2(x.y, x.x)));
        o[0][2] = add2_rn(o[0][2], mulp(pa2, hi2(x)));
        o[0][3] = add2_rn(o[0][3], mulp(pa2, make_float2(x.w, x.z)));
        o[1][0] = add2_rn(o[1][0], mulp(pb2, lo2(x)));
        o[1][1] = add2_rn(o[1][1], mulp(pb2, make_float2(x.y, x.x)));
        o[1][2] = add2_rn(o[1][2], mulp(pb2, hi2(x)));
        o[1][3] = add2_rn(o[1][3], mulp(pb2, make_float2(x.w, x.z)));
      }
    }
  }
  // o[a][0] = (row 2p d0, row 2p+1 d0+1), o[a][1] = (2p d0+1, 2p+1 d0), [2],[3] likewise at d0+2
#pragma unroll
  for (int a = 0; a < 2; a++) {
    const int r0 = 2 * (pa + a);
    if (r0 < ni)
      *reinterpret_cast<float4*>(out + static_cast<int64_t>(rb + i0 + r0) * ldo + h * HD + 4 * dg) =
          make_float4(o[a][0].x, o[a][1].x, o[a][2].x, o[a][3].x);
    if (r0 + 1 < ni)
      *reinterpret_cast<float4*>(out + static_cast<int64_t>(rb + i0 + r0 + 1) * ldo + h * HD + 4 * dg) =
          make_float4(o[a][1].y, o[a][0].y, o[a][3].y, o[a][2].y);
  }
}

__global__ void eval_math_k(int fn, const float* __restrict__ x, float* __restrict__ y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  if (fn == 6) {  // softmax division: y[2i] = x[2i] / x[2i+1] by div_unit_rn, y[2i+1] = x[2i+1]
    const int i0 = i & ~1;
    if (i0 + 1 >= n) { y[i] = v; return; }
    const float b = x[i0 + 1];
    y[i] = (i & 1) ? b : div_unit_rn(x[i0], b, __frcp_rn(b));
    return;
  }
  if (fn >= 4) {  // the packed-pair forms: element i rides in its pair's x or y slot
    const int i0 = i & ~1, i1 = i0 + 1 < n ? i0 + 1 : i0;
    const float2 p = make_float2(x[i0], x[i1]);
    const float2 r = fn == 4 ? tanhf_ref2(p) : gelu_ref2(p);
    y[i] = (i & 1) ? r.y : r.x;
    return;
  }
  y[i] = fn == 0 ? tanhf_ref(v) : fn == 1 ? expf_ref(v) : fn == 2 ? gelu_ref(v) : expm1f_ref(v);
}

// ------------------------------------------------------------------------ launchers
static inline int launched() { return cudaPeekAtLastError() == cudaSuccess ? 0 : -4; }

// Opt a kernel into `bytes` of dynamic shared memory once per (kernel, device).
static void set_smem(const void* kern, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kern, dev})) return;
  // the largest shared-memory carveout, so that as many blocks as fit by shared memory can be
  // resident (the default may size the carveout for one block)
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) ==
          cudaSuccess)
    done.insert({kern, dev});
}

bool kern_prepare() {
  set_smem(reinterpret_cast<const void*>(conv2_k), CV2_SMEM);
  set_smem(reinterpret_cast<const void*>(conv2p_k), CP_SMEM);
  set_smem(reinterpret_cast<const void*>(conv3_k), CV3_SMEM);
  set_smem(reinterpret_cast<const void*>(attn_k), 227 * 1024);
  set_smem(reinterpret_cast<const void*>(gelu_quant_ro_k), 227 * 1024);
  set_smem(reinterpret_cast<const void*>(gelu_quant_cert_k<16>), GQ_WARPS * 2 * 2048 * 4);
  set_smem(reinterpret_cast<const void*>(conv3_cert_k), C3C_SMEM);
  set_smem(reinterpret_cast<const void*>(ln_rows_k), LR_SMEM);
  set_smem(reinterpret_cast<const void*>(ln_quant_k<true>), LnCfg<true>::SMEM);
  return cudaGetLastError() == cudaSuccess;
}

int launch_conv1_w(const float* x, const Conv1W& w, Segs s, int total_frames, float* y1, cudaStream_t st) {
  if (total_frames <= 0) return 0;
  const int n = total_frames * DIM;
  conv1w_k<<<(n + 127) / 128, 128, 0, st>>>(x, w, s, total_frames, y1);
  return launched();
}
int launch_conv1(const float* x, const float* c1, Segs s, int total_frames, float* y1, cudaStream_t st) {
  if (total_frames <= 0) return 0;
  const int n = total_frames * DIM;
  conv1_k<<<(n + 127) / 128, 128, 0, st>>>(x, c1, s, total_frames, y1);
  return launched();
}
// c2t[k][o] = c2[o][k]: the position-pair conv2's weight layout
__global__ void conv2t_pre_k(const float* __restrict__ c2, float* __restrict__ c2t) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= K2 * C2) return;
  const int k = i / C2, o = i - k * C2;
  c2t[i] = c2[static_cast<int64_t>(o) * K2 + k];
}

size_t conv2_prepare_floats() { return static_cast<size_t>(C2) * K2; }
int conv2_prepare(const float* c2, float* c2t, cudaStream_t st) {
  conv2t_pre_k<<<(K2 * C2 + 255) / 256, 256, 0, st>>>(c2, c2t);
  return launched();
}

int launch_conv2(const float* y1, const float* c2, const float* c2t, Segs s, int total_rows, float* y2,
                 cudaStream_t st) {
  if (total_rows <= 0) return 0;
  if (c2t && (reinterpret_cast<uintptr_t>(y1) & 15) == 0 && (reinterpret_cast<uintptr_t>(c2t) & 15) == 0) {
    set_smem(reinterpret_cast<const void*>(conv2p_k), CP_SMEM);
    for (int r0 = 0; r0 < total_rows; r0 += 65535)  // grid.y limit
      conv2p_k<<<dim3(C2 / CP_CH, std::min(65535, total_rows - r0)), TP_THREADS, CP_SMEM, st>>>(y1, c2t, s, r0, y2, -0.0f);
    return launched();
  }
  set_smem(reinterpret_cast<const void*>(conv2_k), CV2_SMEM);
  for (int r0 = 0; r0 < total_rows; r0 += 65535)  // grid.y limit
    conv2_k<<<dim3(C2 / CV2_CH, std::min(65535, total_rows - r0)), TP_THREADS, CV2_SMEM, st>>>(
        y1, c2, s, r0, y2);
  return launched();
}
size_t conv3_cert_prep_floats() { return static_cast<size_t>(K3) * C3 + C3; }
int conv3_cert_prepare(const float* c3, float* prep, cudaStream_t st) {
  conv3_cert_prep_k<<<(K3 * C3 + 255) / 256, 256, 0, st>>>(c3, prep, prep + K3 * C3);
  return launched();
}
int launch_conv3_cert(const float* y2, const float* c3, const float* prep, Segs s, int total_rows, int8_t* xq,
                      float* xs, cudaStream_t st) {
  if (total_rows <= 0) return 0;
  set_smem(reinterpret_cast<const void*>(conv3_cert_k), C3C_SMEM);
  conv3_cert_k<<<(total_rows + C3C_R - 1) / C3C_R, C3C_THREADS, C3C_SMEM, st>>>(y2, c3, prep, prep + K3 * C3, s,
                                                                             total_rows, xq, xs);
  return launched();
}
int launch_conv3(const float* y2, const float* c3, Segs s, int total_rows, float* y3, cudaStream_t st) {
  if (total_rows <= 0) return 0;
  set_smem(reinterpret_cast<const void*>(conv3_k), CV3_SMEM);
  for (int r0 = 0; r0 < total_rows; r0 += 65535)  // grid.y limit
    conv3_k<<<dim3(C3 / CV3_CH, std::min(65535, total_rows - r0)), TP_THREADS, CV3_SMEM, st>>>(
        y2, c3, s, r0, y3);
  return launched();
}
int launch_quant_rows(const float* x, int m, int k, int ldx, int8_t* xq, float* xs, cudaStream_t st) {
  if (m <= 0 || k <= 0) return 0;
  quant_rows_k<<<(m + 7) / 8, 256, 0, st>>>(x, m, k, ldx, nullptr, xq, xs);
  return launched();
}
int launch_quant_rows_max(const float* x, int m, int k, const unsigned* rowmax, int8_t* xq, float* xs,
                          cudaStream_t st) {
  if (m <= 0 || k <= 0) return 0;
  quant_rows_k<<<(m + 7) / 8, 256, 0, st>>>(x, m, k, k, rowmax, xq, xs);
  return launched();
}
int launch_ln_quant(float* h, const float* o, const float* g, const float* b, int m, int8_t* xq, float* xs,
                    cudaStream_t st) {
  if (m <= 0) return 0;
  const int blocks = (m + LN_ROWS - 1) / LN_ROWS;
  if (o) {
    set_smem(reinterpret_cast<const void*>(ln_quant_k<true>), LnCfg<true>::SMEM);
    ln_quant_k<true><<<blocks, LN_THREADS, LnCfg<true>::SMEM, st>>>(h, o, g, b, m, xq, xs);
  } else {
    // two blocks fit an SM: as many rows per block as fill every slot once, at most LR_ROWS
    // (a small M, e.g. one GPU's shard of a multi-GPU job, otherwise leaves SMs idle)
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    const int rpb = std::max(8, std::min(LR_ROWS, (m + 2 * sms - 1) / (2 * sms)));
    const size_t smem = static_cast<size_t>(rpb) * D * 4 + 2 * rpb * 4;
    set_smem(reinterpret_cast<const void*>(ln_rows_k), LR_SMEM);
    ln_rows_k<<<(m + rpb - 1) / rpb, LR_THREADS, smem, st>>>(h, g, b, m, rpb, xq, xs);
  }
  return launched();
}
int launch_gelu_quant(float* x, int m, int k, int8_t* xq, float* xs, cudaStream_t st) {
  if (m <= 0 || k <= 0) return 0;
  gelu_quant_k<<<(m + 7) / 8, 256, 0, st>>>(x, m, k, xq, xs);
  return launched();
}
// GELU + quant of a read-only [m][k] input: the certified kernel for the model's FF width (rows of
// 2048 floats, 16-byte aligned), the all-exact kernel otherwise or when `exact` is set.
int launch_gelu_quant_ro(const float* y, int m, int k, int8_t* xq, float* xs, cudaStream_t st, bool exact) {
  if (m <= 0 || k <= 0) return 0;
  if (!exact && k == 16 * 128 && (reinterpret_cast<uintptr_t>(y) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(xq) & 3) == 0) {
    // persistent warps: as many blocks as are resident at once (two per SM), at most one row each
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      sms = 148;
    constexpr int smem = GQ_WARPS * 2 * 2048 * 4;
    set_smem(reinterpret_cast<const void*>(gelu_quant_cert_k<16>), smem);
    gelu_quant_cert_k<16><<<std::min((m + GQ_WARPS - 1) / GQ_WARPS, 3 * sms), 32 * GQ_WARPS, smem, st>>>(y, m, xq, xs);
    return launched();
  }
  const size_t smem = static_cast<size_t>(GQ_ROWS) * k * sizeof(float);
  if (smem > 227 * 1024) return -2;
  set_smem(reinterpret_cast<const void*>(gelu_quant_ro_k), 227 * 1024);
  gelu_quant_ro_k<<<(m + GQ_ROWS - 1) / GQ_ROWS, 32 * GQ_ROWS, smem, st>>>(y, m, k, xq, xs);
  return launched();
}
int launch_add(float* h, const float* a, size_t n, cudaStream_t st) {
  if (n == 0) return 0;
  const size_t th = (n + 3) / 4;
  add_k<<<static_cast<unsigned>((th + 255) / 256), 256, 0, st>>>(h, a, n);
  return launched();
}
int launch_argmax_rows(const float* x, int m, int n, uint32_t* out, cudaStream_t st) {
  if (m <= 0 || n <= 0) return 0;
  argmax_k<<<m, 256, 0, st>>>(x, n, out);
  return launched();
}
int launch_keys_to_ids(const unsigned long long* keys, int m, uint32_t* ids, cudaStream_t st) {
  if (m <= 0) return 0;
  keys_to_ids_k<<<(m + 255) / 256, 256, 0, st>>>(keys, m, ids);
  return launched();
}
int launch_attention(const float* q, const float* k, const float* v, int ld, Segs s, const int* toff,
                     const int* tord, int total_tiles, int max_t1, float* out, int ldo, cudaStream_t st) {
  if (total_tiles <= 0) return 0;
  const size_t smem = attention_smem_bytes(max_t1);
  if (smem > 227 * 1024) return -2;
  set_smem(reinterpret_cast<const void*>(attn_k), 227 * 1024);  // the largest opt-in size; each launch passes its own
  attn_k<<<dim3(total_tiles, HEADS), 256, smem, st>>>(q, k, v, ld, s, toff, tord, max_t1, out, ldo);
  return launched();
}

}  // namespace wasr

// ============================================================================ wk_* C ABI
using namespace wasr;

static Segs one_seg(int t, int t1) {
  Segs s{};
  s.n = 1;
  s.t0 = t;
  s.t10 = t1;
  return s;
}

extern "C" {

const char* wk_version(void) { return "wasr-b200 wk 1.0 (sm_100a; exact-order conv/LN/quant; fused attention)"; }

void wk_front(void* stream, const float* x, const float* c1, const float* c2, const float* c3, int t, int t1,
              float* y1, float* y2, float* y3) {
  if (!x || !c1 || !c2 || !c3 || !y1 || !y2 || !y3 || t <= 0 || t1 <= 0) return;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const Segs s = one_seg(t, t1);
  launch_conv1(x, c1, s, t, y1, st);
  launch_conv2(y1, c2, nullptr, s, t1, y2, st);
  launch_conv3(y2, c3, s, t1, y3, st);
}

// the 512-wide kernel moves rows as float4 / char4
static bool ln_aligned(const float* h, const float* o, const float* g, const float* b, const int8_t* xq) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(o) |
                      reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(b);
  return (a & 15) == 0 && (reinterpret_cast<uintptr_t>(xq) & 3) == 0;
}

void wk_norm_quant(void* stream, const float* h, const float* g, const float* b, int t, int d, int8_t* xq,
                   float* xs) {
  if (!h || !g || !b || !xq || !xs || t <= 0 || d <= 0) return;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d == D && ln_aligned(h, h, g, b, xq))
    launch_ln_quant(const_cast<float*>(h), nullptr, g, b, t, xq, xs, st);
  else
    ln_quant_any_k<<<t, 256, 0, st>>>(const_cast<float*>(h), nullptr, g, b, d, xq, xs);
}

void wk_add_norm_quant(void* stream, float* h, const float* o, const float* g, const float* b, int t, int d,
                       int8_t* xq, float* xs) {
  if (!h || !o || !g || !b || !xq || !xs || t <= 0 || d <= 0) return;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (d == D && ln_aligned(h, o, g, b, xq))
    launch_ln_quant(h, o, g, b, t, xq, xs, st);
  else
    ln_quant_any_k<<<t, 256, 0, st>>>(h, o, g, b, d, xq, xs);
}

void wk_quant(void* stream, const float* x, int t, int k, int8_t* xq, float* xs) {
  if (!x || !xq || !xs) return;
  launch_quant_rows(x, t, k, k, xq, xs, static_cast<cudaStream_t>(stream));
}

void wk_gelu_quant(void* stream, float* x, int t, int k, int8_t* xq, float* xs) {
  if (!x || !xq || !xs) return;
  launch_gelu_quant(x, t, k, xq, xs, static_cast<cudaStream_t>(stream));
}

void wk_add(void* stream, float* h, const float* a, int t, int d) {
  if (!h || !a || t <= 0 || d <= 0) return;
  launch_add(h, a, static_cast<size_t>(t) * d, static_cast<cudaStream_t>(stream));
}

void wk_argmax(void* stream, const float* x, int t, int n, uint32_t* out) {
  if (!x || !out) return;
  launch_argmax_rows(x, t, n, out, static_cast<cudaStream_t>(stream));
}

int wk_last_error(void) { return static_cast<int>(cudaGetLastError()); }

// csrc/wk_attention_*.cu return codes: -1 null pointer, -2 bad shape, -3 head dim != 64.
static int attention_abi(void* stream, const float* q, const float* k, const float* v, int t, int d, int heads,
                         float* out) {
  if (!q || !k || !v || !out) return -1;
  if (t <= 0) return 0;
  if (heads <= 0 || d % heads != 0) return -2;
  if (d / heads != HD) return -3;
  if (heads != HEADS) return -2;
  if (attention_smem_bytes(t) > 227 * 1024) return -2;
  const Segs s = one_seg(t * 5, t);  // only the row count matters to attention
  return launch_attention(q, k, v, d, s, nullptr, nullptr, (t + ATT_QT - 1) / ATT_QT, t, out, d,
                          static_cast<cudaStream_t>(stream));
}

int wk_attention_fast(void* stream, const float* q, const float* k, const float* v, int t, int d, int heads,
                      float* scratch, float* out) {
  (void)scratch;
  return attention_abi(stream, q, k, v, t, d, heads, out);
}

void wk_attention(void* stream, const float* q, const float* k, const float* v, int t, int d, int heads,
                  float* scratch, float* out) {
  (void)scratch;
  attention_abi(stream, q, k, v, t, d, heads, out);
}

int wk_attention_tiled(void* stream, const float* q, const float* k, const float* v, int t, int d, int heads,
                       float* scratch, float* out) {
  (void)scratch;
  return attention_abi(stream, q, k, v, t, d, heads, out);
}

int wk_attention_tiled_tuned(void* stream, const float* q, const float* k, const float* v, int t, int d, int heads,
                             float* out, int it, int ch) {
  if (it != 8 && it != 16 && it != 32 && it != 64) return -4;  // same accepted set as the reference
  (void)ch;
  return attention_abi(stream, q, k, v, t, d, heads, out);
}

const char* wk_attention_tiled_version(void) {
  return "wk_attention_tiled (wasr-b200 sm_100a fused fp32, 32-query tiles, hd=64)";
}

int wk_attention_cublas(void* stream, const float* q, const float* k, const float* v, int t, int d, int heads,
                        float* scratch, float* out) {
  if (!scratch) return -1;  // the reference requires the scratch buffer on this entry point
  return attention_abi(stream, q, k, v, t, d, heads, out);
}

int wk_attention_cublas_part(int part, void* stream, const float* q, const float* k, const float* v, int t, int d,
                             int heads, float* scratch, float* out) {
  (void)scratch;
  if (part == 0 || part == 1) return 0;
  return attention_abi(stream, q, k, v, t, d, heads, out);
}

// Parity hook for the certified conv3 + quant: prep = conv3_cert_prep_floats() floats (filled
// here from c3), roff = device row offsets of nseg segments or nullptr for one segment of `rows`.
int wasr_conv3_quant(const float* y2, const float* c3, float* prep, const int* roff, int nseg, int rows, int8_t* xq,
                     float* xs, void* stream) {
  if (!y2 || !c3 || !prep || !xq || !xs || rows < 0 || (roff && nseg <= 0)) return -1;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (conv3_cert_prepare(c3, prep, st) != 0) return -4;
  Segs s{};
  s.foff = nullptr;
  s.roff = roff;
  s.n = roff ? nseg : 1;
  s.t0 = 0;
  s.t10 = rows;
  return launch_conv3_cert(y2, c3, prep, s, rows, xq, xs, st);
}

// Parity hook for conv1: by_value = 1 runs the engine's kernel (the weights copied to the host
// here and passed by value; this call waits for that copy), 0 the reference ABI's (weights read
// from device memory).  foff = device frame offsets of nseg windows, or nullptr for one window.
int wasr_conv1(const float* x, const float* c1, const int* foff, int nseg, int frames, int by_value, float* y1,
               void* stream) {
  if (!x || !c1 || !y1 || frames < 0 || (foff && nseg <= 0)) return -1;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  Segs s{};
  s.foff = foff;
  s.roff = nullptr;
  s.n = foff ? nseg : 1;
  s.t0 = frames;
  s.t10 = 0;
  if (!by_value) return launch_conv1(x, c1, s, frames, y1, st);
  Conv1W w;
  if (cudaMemcpyAsync(w.w, c1, sizeof(w.w), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return -4;
  return launch_conv1_w(x, w, s, frames, y1, st);
}

// Parity hook for conv2: c2t = conv2_prepare_floats() floats (filled here from c2) selects the
// engine's position-pair kernel, nullptr the reference ABI's; foff / roff = device frame / row
// offsets of nseg windows, or both nullptr for one window of `frames` frames and `rows` rows.
int wasr_conv2(const float* y1, const float* c2, float* c2t, const int* foff, const int* roff, int nseg, int frames,
               int rows, float* y2, void* stream) {
  if (!y1 || !c2 || !y2 || rows < 0 || frames < 0 || (!foff != !roff) || (roff && nseg <= 0)) return -1;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (c2t && conv2_prepare(c2, c2t, st) != 0) return -4;
  Segs s{};
  s.foff = foff;
  s.roff = roff;
  s.n = roff ? nseg : 1;
  s.t0 = frames;
  s.t10 = rows;
  return launch_conv2(y1, c2, c2t, s, rows, y2, st);
}

// Parity hooks for the certified GELU + quant: the engine's kernel choice (exact = 0) or the
// all-exact kernel (exact = 1) on a read-only [m][k] input; and the exhaustive bound scan.
int wasr_gelu_quant(const float* y, int m, int k, int8_t* xq, float* xs, int exact, void* stream) {
  if (!y || !xq || !xs) return -1;
  return launch_gelu_quant_ro(y, m, k, xq, xs, static_cast<cudaStream_t>(stream), exact != 0);
}
int wasr_gelu_cert_scan(unsigned long long start, unsigned long long count, unsigned long long* stats,
                        void* stream) {
  if (!stats || start + count > (1ull << 32) || (start | count) & 1) return -1;
  if (count == 0) return 0;
  gelu_cert_scan_k<<<148 * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(start, count, stats);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

// Parity hook: evaluate the device restatements of the libm functions the reference calls
// (fn 0 tanhf, 1 expf, 2 the GELU of src/model.rs:710-712, 3 expm1f; 4 tanhf and 5 the GELU
// in their packed two-element forms; 6 the softmax division of (x[2i], x[2i+1])) over n floats.
int wasr_eval_math(int fn, const float* x, float* y, int n, void* stream) {
  if (!x || !y || fn < 0 || fn > 6) return -1;
  if (n <= 0) return 0;
  eval_math_k<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(fn, x, y, n);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

const char* wk_attention_version(void) {
  return "wk_attention (wasr-b200 sm_100a: one fused kernel; scores stay on chip; hd=64)";
}

}  // extern "C"
