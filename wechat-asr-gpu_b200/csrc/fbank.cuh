// fbank.cuh -- HTK-style log-mel fbank of src/fbank.rs: the tables, the host frame function
// and the device entry points.  25 ms Hamming window, pre-emphasis 0.97, f64 radix-2 FFT512,
// 39 HTK mel bands + log energy, CMS over the last 50 frames.  Host and device evaluate the same
// operations in the same order (the host code is compiled without floating-point contraction;
// the device code uses explicitly rounded f64 intrinsics), from the same tables.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <utility>

namespace fb {

constexpr int WIN = 400, HOP = 160, NFFT = 512, NCH = 39, CMS_WIN = 50, FDIM = NCH + 1;

struct Tables {
  double ham[WIN];
  double twr[NFFT / 2], twi[NFFT / 2];
  int lo[NFFT / 2], hi[NFFT / 2];
  double wl[NFFT / 2], wh[NFFT / 2];
  Tables() {
    const double pi = 3.14159265358979323846;
    for (int i = 0; i < WIN; i++) ham[i] = 0.54 - 0.46 * std::cos(2.0 * pi * static_cast<double>(i) / (WIN - 1));
    for (int i = 0; i < NFFT / 2; i++) {
      const double a = -2.0 * pi * static_cast<double>(i) / NFFT;
      twr[i] = std::cos(a);
      twi[i] = std::sin(a);
    }
    auto mel = [](double f) { return 1127.0 * std::log(1.0 + f / 700.0); };
    const double top = mel(8000.0);
    double cf[NCH + 1];
    for (int i = 1; i <= NCH + 1; i++) cf[i - 1] = top * static_cast<double>(i) / (NCH + 1);
    for (int k = 1; k <= NFFT / 2; k++) {
      const double mv = mel(static_cast<double>(k) * 16000.0 / NFFT);
      int c = 0;
      while (c < NCH + 1 && cf[c] < mv) c++;
      const int x = k - 1;
      lo[x] = hi[x] = 0;
      wl[x] = wh[x] = 0.0;
      if (c == 0) {
        wl[x] = mv / cf[0];
      } else if (c < NCH) {
        const double w = (cf[c] - mv) / (cf[c] - cf[c - 1]);
        lo[x] = c - 1;
        wl[x] = w;
        hi[x] = c;
        wh[x] = 1.0 - w;
      } else if (c == NCH) {
        lo[x] = NCH - 1;
        wl[x] = (cf[NCH] - mv) / (cf[NCH] - cf[NCH - 1]);
      }
    }
  }
};

inline const Tables& tables() {
  static const Tables T;
  return T;
}

inline void frame(const int16_t* x, double* out) {
  const Tables& T = tables();
  double re[NFFT] = {0}, im[NFFT] = {0};
  double e = 0.0;
  for (int i = 0; i < WIN; i++) {
    const double v = x[i];
    e += v * v;
    const double pe = i == 0 ? v * (1.0 - 0.97) : v - 0.97 * static_cast<double>(x[i - 1]);
    re[i] = pe * T.ham[i];
  }
  for (int i = 1, j = 0; i < NFFT; i++) {
    int b = NFFT >> 1;
    while (j & b) {
      j ^= b;
      b >>= 1;
    }
    j |= b;
    if (i < j) {
      std::swap(re[i], re[j]);
      std::swap(im[i], im[j]);
    }
  }
  for (int len = 2; len <= NFFT; len <<= 1) {
    const int step = NFFT / len;
    for (int s = 0; s < NFFT; s += len)
      for (int k = 0; k < len / 2; k++) {
        const double wr = T.twr[k * step], wi = T.twi[k * step];
        const int a = s + k, b = s + k + len / 2;
        const double tr = re[b] * wr - im[b] * wi;
        const double ti = re[b] * wi + im[b] * wr;
        re[b] = re[a] - tr;
        im[b] = im[a] - ti;
        re[a] += tr;
        im[a] += ti;
      }
  }
  for (int i = 0; i < FDIM; i++) out[i] = 0.0;
  for (int k = 0; k < NFFT / 2; k++) {
    const double p = re[k + 1] * re[k + 1] + im[k + 1] * im[k + 1];
    out[T.lo[k]] += p * T.wl[k];
    out[T.hi[k]] += p * T.wh[k];
  }
  for (int i = 0; i < NCH; i++) out[i] = std::log(out[i] > 1.0 ? out[i] : 1.0);
  out[NCH] = std::log(e > 1e-10 ? e : 1e-10);
}

}  // namespace fb

namespace fb {
// Batched fbank on the GPU (csrc/fbank.cu): utterance i has samples [soff[i], soff[i+1]) of pcm
// and frames [foff[i], foff[i+1]) of the outputs (foff = prefix of (n_i - 400) / 160 + 1, 0 for
// n_i < 400).  raw: [frames][40] f64 scratch; feats: [frames][40] f32; sil: [n][40] f32 (the
// normalised silence frame of each utterance).  All pointers are device pointers.
int fbank_device(const int16_t* pcm, const int64_t* soff, const int64_t* foff, int n, int64_t frames,
                 double* raw, float* feats, float* sil, cudaStream_t st);
}  // namespace fb
