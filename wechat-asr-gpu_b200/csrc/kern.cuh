// kern.cuh -- non-GEMM kernels of the window forward, written segment-aware so that one
// launch serves either one window (the reference ABI, t <= TMAX) or many stacked windows
// of different lengths (the batched engine).
//
// A "segment" is one window: frames [foff, foff+t) of the stacked feature array and output
// rows [roff, roff+t1) of every activation, t1 = (t-5)/5+1.  The time axis of the conv
// frontend and the keys of attention never cross a segment boundary.
#pragma once

#include "common.cuh"

namespace wasr {

struct Segs {
  const int* foff;  // [n+1] frame prefix offsets (device), or nullptr for one inline segment
  const int* roff;  // [n+1] row prefix offsets (device)
  int n;
  int t0, t10;      // the inline segment (foff == nullptr)

  __device__ __forceinline__ int frame_begin(int w) const { return foff ? foff[w] : 0; }
  __device__ __forceinline__ int frames(int w) const { return foff ? foff[w + 1] - foff[w] : t0; }
  __device__ __forceinline__ int row_begin(int w) const { return roff ? roff[w] : 0; }
  __device__ __forceinline__ int rows(int w) const { return roff ? roff[w + 1] - roff[w] : t10; }
  // segment holding output row r (last w with roff[w] <= r; skips empty segments)
  __device__ __forceinline__ int seg_of_row(int r) const {
    if (!roff) return 0;
    int lo = 0, hi = n - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (roff[mid] <= r) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
  __device__ __forceinline__ int seg_of_frame(int g) const {
    if (!foff) return 0;
    int lo = 0, hi = n - 1;
    while (lo < hi) {
      int mid = (lo + hi + 1) >> 1;
      if (foff[mid] <= g) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
};

// host launchers (stream-ordered, no allocation); return 0 or -4 on launch failure
int launch_conv1(const float* x, const float* c1, Segs s, int total_frames, float* y1, cudaStream_t st);
// conv1 with its 32 x 25 weights passed by value (a kernel argument): every product reads its
// weight from the constant bank, no shared-memory loads.  Same results as launch_conv1.
struct Conv1W {
  float w[C1 * 25];
};
int launch_conv1_w(const float* x, const Conv1W& w, Segs s, int total_frames, float* y1, cudaStream_t st);
// c2t: the conv2 weights transposed to [tap][out] by conv2_prepare (conv2_prepare_floats()
// floats), which selects the position-pair kernel; nullptr stages the weights from c2's
// [out][tap] layout (the reference ABI's wk_front).
int launch_conv2(const float* y1, const float* c2, const float* c2t, Segs s, int total_rows, float* y2,
                 cudaStream_t st);
int launch_conv3(const float* y2, const float* c3, Segs s, int total_rows, float* y3, cudaStream_t st);
size_t conv2_prepare_floats();
int conv2_prepare(const float* c2, float* c2t, cudaStream_t st);
// conv3 fused with the certified row quantisation of its output (the engine's path): the int8
// rows and scales equal quant(conv3(y2)) of the reference order; prep holds the transposed
// weights and weight norms (conv3_cert_prepare, conv3_cert_prep_floats() floats)
size_t conv3_cert_prep_floats();
int conv3_cert_prepare(const float* c3, float* prep, cudaStream_t st);
int launch_conv3_cert(const float* y2, const float* c3, const float* prep, Segs s, int total_rows, int8_t* xq,
                      float* xs, cudaStream_t st);
int launch_quant_rows(const float* x, int m, int k, int ldx, int8_t* xq, float* xs, cudaStream_t st);
int launch_quant_rows_max(const float* x, int m, int k, const unsigned* rowmax, int8_t* xq, float* xs,
                          cudaStream_t st);
int launch_ln_quant(float* h, const float* o, const float* g, const float* b, int m, int8_t* xq, float* xs,
                    cudaStream_t st);
int launch_gelu_quant(float* x, int m, int k, int8_t* xq, float* xs, cudaStream_t st);
// GELU + per-row quant of a read-only input (the GELU values are not written back)
int launch_gelu_quant_ro(const float* y, int m, int k, int8_t* xq, float* xs, cudaStream_t st, bool exact = false);
int launch_add(float* h, const float* a, size_t n, cudaStream_t st);
int launch_argmax_rows(const float* x, int m, int n, uint32_t* out, cudaStream_t st);
int launch_keys_to_ids(const unsigned long long* keys, int m, uint32_t* ids, cudaStream_t st);
// attention over segments; q/k/v rows of stride ld floats (head h at column h*64).
// toff: [n+1] prefix of per-segment query tiles (ceil(t1/ATT_QT)), or nullptr for the inline
// segment; tord: optional [total_tiles] launch order of the tiles (longest segments first);
// max_t1 bounds every segment's length (sizes the on-chip score tile).
constexpr int ATT_QT = 64;
int launch_attention(const float* q, const float* k, const float* v, int ld, Segs s, const int* toff,
                     const int* tord, int total_tiles, int max_t1, float* out, int ldo, cudaStream_t st);
size_t attention_smem_bytes(int max_t1);
// Set the kernels' shared-memory attributes on the current device (call outside capture).
bool kern_prepare();

}  // namespace wasr
