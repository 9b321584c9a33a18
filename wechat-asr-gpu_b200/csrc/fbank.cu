// fbank.cu -- the fbank of src/fbank.rs:79-156 on the GPU, batched over utterances.
//
// frame_k: 4 frames per 256-thread block, 64 threads per frame.  The 400 windowed samples go
// straight to their bit-reversed slots (the reference's swap loop is the bit-reversal
// involution), the nine radix-2 stages run four butterflies per thread with the reference's
// expressions (tr = re[b]*wr - im[b]*wi, ti = re[b]*wi + im[b]*wr, re[b] = re[a]-tr, ...), each product and
// sum explicitly rounded in f64.  The frame energy sum(v*v) is a sum of integers below 2^53, so
// it is exact in any order.  Each mel channel folds its non-zero weights in bin order (the
// reference adds its zero weights too; adding +0.0 to a non-negative sum changes nothing).
// The log is CUDA's double log (within one unit in the last place of the host libm's; the f32
// features that follow round those f64 values, so they agree unless an f64 value sits within
// an f64 ulp of an f32 rounding boundary); log(1e-10) comes from the host libm.
// cms_k: one thread per (utterance, dimension) runs the 50-frame rolling mean in frame order
// (src/fbank.rs:143-152) and writes the f32 features and the normalised silence frame.
#include <cstdio>
#include <mutex>
#include <vector>

#include "../../include/wasr.h"
#include "common.cuh"
#include "fbank.cuh"

namespace fb {

struct DevTables {
  double ham[WIN];
  double twr[NFFT / 2], twi[NFFT / 2];
  int cstart[NCH + 1];   // channel c's weights: [cstart[c], cstart[c+1]) of ck / cw, bin order
  int ck[NFFT];
  double cw[NFFT];
  double log_floor;      // log(1e-10) as the host libm gives it (silent frames, the silence frame)
};
// in global memory, read through the read-only cache: the lanes of a warp index the tables
// at different places, which the constant cache would serialise
__device__ DevTables kT;

// Upload the tables once per device.
static bool ensure_tables() {
  static std::mutex mu;
  static unsigned done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (done & (1u << (dev & 31))) return true;
  const Tables& T = tables();
  DevTables d{};
  for (int i = 0; i < WIN; i++) d.ham[i] = T.ham[i];
  for (int i = 0; i < NFFT / 2; i++) {
    d.twr[i] = T.twr[i];
    d.twi[i] = T.twi[i];
  }
  int n = 0;
  for (int c = 0; c < NCH; c++) {
    d.cstart[c] = n;
    for (int k = 0; k < NFFT / 2; k++) {  // the order of the reference loop: lo slot, then hi slot
      if (T.lo[k] == c && T.wl[k] != 0.0) { d.ck[n] = k; d.cw[n] = T.wl[k]; n++; }
      if (T.hi[k] == c && T.wh[k] != 0.0) { d.ck[n] = k; d.cw[n] = T.wh[k]; n++; }
    }
  }
  d.cstart[NCH] = n;
  d.log_floor = std::log(1e-10);
  if (cudaMemcpyToSymbol(kT, &d, sizeof(d)) != cudaSuccess) return false;
  done |= 1u << (dev & 31);
  return true;
}

constexpr int FPB = 4;  // frames per block, 64 threads each

__global__ void __launch_bounds__(256) frame_k(const int16_t* __restrict__ pcm, const int64_t* __restrict__ soff,
                                               const int64_t* __restrict__ foff, int n, int64_t frames,
                                               double* __restrict__ raw) {
  __shared__ double re[FPB][NFFT], im[FPB][NFFT], pw[FPB][NFFT / 2];
  __shared__ double esum[FPB][2];
  const int fr = threadIdx.x >> 6, t = threadIdx.x & 63;
  const int64_t f = static_cast<int64_t>(blockIdx.x) * FPB + fr;
  const bool live = f < frames;  // dead frames still take part in the barriers
  double* R = re[fr];
  double* I = im[fr];
  double e = 0.0;
  if (live) {
    int lo = 0, hi = n - 1;  // utterance holding frame f (last i with foff[i] <= f)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (foff[mid] <= f) lo = mid; else hi = mid - 1;
    }
    const int16_t* x = pcm + soff[lo] + (f - foff[lo]) * HOP;
    for (int i = t; i < NFFT; i += 64) {
      const int slot = static_cast<int>(__brev(static_cast<unsigned>(i)) >> 23);
      double v = 0.0;
      if (i < WIN) {
        const double xv = x[i];
        e = __dadd_rn(e, __dmul_rn(xv, xv));
        const double pe =
            i == 0 ? __dmul_rn(xv, 1.0 - 0.97) : __dsub_rn(xv, __dmul_rn(0.97, static_cast<double>(x[i - 1])));
        v = __dmul_rn(pe, __ldg(&kT.ham[i]));
      }
      R[slot] = v;
      I[slot] = 0.0;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);  // integer-valued: exact
  if ((t & 31) == 0) esum[fr][t >> 5] = e;
  __syncthreads();
#pragma unroll 1
  for (int len = 2; len <= NFFT; len <<= 1) {
    const int half = len >> 1;
    if (live) {
#pragma unroll
      for (int r = 0; r < 4; r++) {  // butterflies t, t+64, t+128, t+192 of this stage
        const int bi = t + 64 * r, k = bi & (half - 1), a = (bi / half) * len + k, b = a + half;
        const double wr = __ldg(&kT.twr[k * (NFFT / len)]), wi = __ldg(&kT.twi[k * (NFFT / len)]);
        const double rb = R[b], ib = I[b], ra = R[a], ia = I[a];
        const double tr = __dsub_rn(__dmul_rn(rb, wr), __dmul_rn(ib, wi));
        const double ti = __dadd_rn(__dmul_rn(rb, wi), __dmul_rn(ib, wr));
        R[b] = __dsub_rn(ra, tr);
        I[b] = __dsub_rn(ia, ti);
        R[a] = __dadd_rn(ra, tr);
        I[a] = __dadd_rn(ia, ti);
      }
    }
    __syncthreads();
  }
  if (live) {
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int kk = t + 64 * r;
      pw[fr][kk] = __dadd_rn(__dmul_rn(R[kk + 1], R[kk + 1]), __dmul_rn(I[kk + 1], I[kk + 1]));
    }
  }
  __syncthreads();
  if (!live) return;
  double* out = raw + f * FDIM;
  if (t < NCH) {
    double s = 0.0;
    const int j1 = __ldg(&kT.cstart[t + 1]);
    for (int j = __ldg(&kT.cstart[t]); j < j1; j++) s = __dadd_rn(s, __dmul_rn(pw[fr][__ldg(&kT.ck[j])], __ldg(&kT.cw[j])));
    out[t] = log(s > 1.0 ? s : 1.0);
  } else if (t == NCH) {
    const double es = esum[fr][0] + esum[fr][1];
    out[NCH] = es > 1e-10 ? log(es) : __ldg(&kT.log_floor);
  }
}

__global__ void cms_k(const double* __restrict__ raw, const int64_t* __restrict__ foff, int n, float* __restrict__ feats,
                      float* __restrict__ sil) {
  const int u = blockIdx.x * 2 + (threadIdx.x >= 64 ? 1 : 0), i = threadIdx.x & 63;
  if (u >= n || i >= FDIM) return;
  const int64_t f0 = foff[u], nf = foff[u + 1] - f0;
  double sum = 0.0;
  int hn = 0;
  for (int64_t k = 0; k < nf; k++) {
    const double v = raw[(f0 + k) * FDIM + i];
    if (hn == CMS_WIN) {
      sum = __dsub_rn(sum, raw[(f0 + k - CMS_WIN) * FDIM + i]);
      hn--;
    }
    hn++;
    sum = __dadd_rn(sum, v);
    feats[(f0 + k) * FDIM + i] = __double2float_rn(__dsub_rn(v, __ddiv_rn(sum, static_cast<double>(hn))));
  }
  const double s = i == NCH ? __ldg(&kT.log_floor) : 0.0;
  sil[static_cast<int64_t>(u) * FDIM + i] =
      __double2float_rn(__dsub_rn(s, __ddiv_rn(sum, static_cast<double>(hn > 0 ? hn : 1))));
}

int fbank_device(const int16_t* pcm, const int64_t* soff, const int64_t* foff, int n, int64_t frames, double* raw,
                 float* feats, float* sil, cudaStream_t st) {
  if (n <= 0) return 0;
  if (!pcm || !soff || !foff || !raw || !feats || !sil) return -1;
  if (!ensure_tables()) return -4;
  if (frames > 0) frame_k<<<static_cast<unsigned>((frames + FPB - 1) / FPB), 256, 0, st>>>(pcm, soff, foff, n, frames, raw);
  cms_k<<<(n + 1) / 2, 128, 0, st>>>(raw, foff, n, feats, sil);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace fb

extern "C" int wasr_fbank_device(const int16_t* pcm, const int64_t* soff, const int64_t* foff, int n,
                                 int64_t frames, double* raw, float* feats, float* sil, void* stream) {
  return fb::fbank_device(pcm, soff, foff, n, frames, raw, feats, sil, static_cast<cudaStream_t>(stream));
}
