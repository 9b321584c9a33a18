/* wasr.h -- additive C ABI of the B200 batch-transcription engine (libwasr_gpu.so).
 *
 * These entry points have no one-to-one counterpart in the reference ABI: they are the
 * "new-build additions" layered on top of the reference's wp_* / wk_* calls (which are
 * declared, unchanged, in wtlgpu.h).  They cover:
 *   - the weight-blob plan (which byte offset holds which tensor), mirroring the
 *     reference's Plan / PlanLayer / PlanQ structs (src/model.rs:58-94) and the blob
 *     packer build_plan (src/model.rs:148-237);
 *   - a whole-model batched, ragged forward: many windows stacked into one set of
 *     GEMMs (the reference runs one window at a time: Model::run_gpu, src/model.rs:546-619);
 *   - batch transcription with the reference's window schedule (Stream::push/commit/
 *     finish, src/stream.rs:58-168) driven round by round across utterances;
 *   - the HTK fbank of src/fbank.rs on the host (feature extraction for the schedule);
 *   - per-output-channel weight scales and device selection.
 *
 * Model constants follow src/model.rs:21-32.
 */
#ifndef WASR_H
#define WASR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WASR_D 512          /* model width */
#define WASR_HEADS 8
#define WASR_HD 64          /* head dim */
#define WASR_FF 2048
#define WASR_DIM 40         /* fbank feature dim (39 log-mel + log-energy) */
#define WASR_C1 32          /* conv channels */
#define WASR_C2 64
#define WASR_C3 192
#define WASR_W2 41          /* conv2 output width (40 + one zero column) */
#define WASR_FLAT 3840      /* 192 * 20 */
#define WASR_MAX_LAYERS 40
#define WASR_NONE ((uint64_t)-1)

/* Stream schedule defaults (src/stream.rs:11-18). */
#define WASR_PREV 200
#define WASR_POST 100
#define WASR_PAD 50
#define WASR_WHOLE_MAX 2000

/* One int8 weight matrix [n][k] (row-major = K-major) inside the blob.
 * `s` is the per-tensor scale the reference keeps (src/xnet.rs:70, PlanQ src/model.rs:60-63).
 * `scale_off` != WASR_NONE points at an fp32 [n] per-output-channel scale vector, which then
 * replaces `s` in the epilogue:  out = (acc * xs[i]) * ws[j] + bias[j]. */
typedef struct WasrMat {
  uint64_t off;
  uint64_t scale_off;
  float s;
  int32_t n;
  int32_t k;
  int32_t reserved;
} WasrMat;

/* One encoder layer (PlanLayer, src/model.rs:66-79).  qb/kb/vb/ob are optional projection
 * biases (WASR_NONE in the reference model, which has none: src/model.rs:526-531). */
typedef struct WasrLayer {
  uint64_t pn_g, pn_b, mn_g, mn_b;
  WasrMat q, k, v, o, f1, f2;
  uint64_t qb, kb, vb, ob, f1b, f2b;
} WasrLayer;

/* Whole model (Plan, src/model.rs:81-94).  out.n = out_n = vocab rounded up to a multiple
 * of 4, with zero weight rows and -1e30 bias in the padding (src/model.rs:229-231). */
typedef struct WasrPlan {
  int32_t n_layers;
  int32_t vocab;
  int32_t out_n;
  int32_t reserved;
  WasrMat lin, out;
  uint64_t lin_b, out_b, c1, c2, c3;
  WasrLayer layers[WASR_MAX_LAYERS];
} WasrPlan;

typedef struct WasrModel WasrModel;

/* Upload the blob to `device` and size activation buffers for up to `max_rows` stacked
 * output frames (t1 rows) per batched forward.  Returns NULL on failure. */
WasrModel* wasr_model_create(const void* blob, size_t bytes, const WasrPlan* plan, int device,
                             int max_rows);
void wasr_model_destroy(WasrModel* m);
/* Stream every later call of this model runs on (NULL = the model's own stream). */
int wasr_model_set_stream(WasrModel* m, void* stream);
void* wasr_model_stream(WasrModel* m);
/* Enable (1) / disable (0) CUDA-graph capture and replay of whole batched forwards. */
int wasr_model_set_graphs(WasrModel* m, int on);
/* Most recent device-side error word (0 = none); a nonzero value means a bounded wait in a
 * kernel gave up.  Cleared by reading. */
int wasr_model_error(WasrModel* m);

#define WASR_F_DEVICE 1   /* feats / ids / logits pointers are device pointers */
#define WASR_F_NOSYNC 2   /* do not synchronise the stream before returning (device mode) */

/* Per-kernel timing.  With profiling on, every kernel the engine enqueues is bracketed by a
 * pair of CUDA events on the model's stream (captured into the CUDA graphs as event nodes), so
 * the timing is taken inside the real, graph-replayed run.  wasr_model_profile() sums, per
 * kernel class, the durations of the most recent execution of every cached graph (plus the
 * last eager chunk).  Turning profiling on or off drops the cached graphs. */
enum {
  WASR_K_CONV1 = 0, WASR_K_CONV2, WASR_K_CONV3, WASR_K_QUANT, WASR_K_GEMM_LIN, WASR_K_LN,
  WASR_K_GEMM_QKV, WASR_K_ATTN, WASR_K_GEMM_O, WASR_K_GEMM_F1, WASR_K_GEMM_F2, WASR_K_GEMM_OUT,
  WASR_K_IDS, WASR_K_GELU, WASR_K_COUNT
};
int wasr_model_set_profile(WasrModel* m, int on);
int wasr_model_profile(WasrModel* m, double* ms, int64_t* launches, int ncat);
/* Kernels launched by this model so far (a graph replay counts every kernel it holds). */
int64_t wasr_model_kernel_launches(WasrModel* m);

/* Batched ragged forward (Model::forward on n_win windows at once, src/model.rs:368-386):
 *   feats  : [sum t][40] fp32, windows concatenated
 *   t      : [n_win] frames per window (host array); t < 5 gives zero output frames
 *   ids    : [sum t1] uint32 argmax token ids, t1 = (t-5)/5+1
 *   logits : optional [sum t1][out_n] fp32 (debug/parity); NULL = fused GEMM+argmax only
 * Returns 0 or a negative error code. */
int wasr_forward(WasrModel* m, const float* feats, const int32_t* t, int n_win, uint32_t* ids,
                 float* logits, int flags);

/* Batch transcription with the reference stream schedule (src/stream.rs:58-168): every
 * utterance runs its own commit/finish sequence; the k-th windows of all utterances are
 * stacked into one wasr_forward.
 *   feats    : [sum n_frames][40] host fp32 (CMS-normalised fbank frames)
 *   sil      : [n_utt][40] host fp32 silence frame of each utterance (Fbank::silence)
 *   ids      : output per-frame token ids (before CTC collapse), utterances concatenated
 *   ids_off  : [n_utt+1] offsets into ids
 * Returns 0, or a negative code (-20: ids_cap too small). */
int wasr_transcribe(WasrModel* m, const float* feats, const int64_t* n_frames, const float* sil,
                    int n_utt, int prev, int blk, int post, uint32_t* ids, int64_t* ids_off,
                    int64_t ids_cap);

/* wasr_transcribe with the features already on the GPU, e.g. wasr_fbank_device's output (no
 * counterpart in the reference, whose fbank and window assembly run on the host,
 * src/stream.rs:128-147).  feats [sum n_frames][40] and sil [n_utt][40] are device pointers on
 * the model's device; n_frames, ids and ids_off are host arrays.  Each round's windows (frames
 * plus the silence pad) are gathered on the device into a staging buffer the model keeps and
 * grows, so the features never cross to the host; a round of whole utterances laid out back to
 * back is read straight from feats.  Work already queued that writes feats or sil must be
 * complete or ordered before the call (it runs on the model's stream).  Same ids, ids_off and
 * return codes as wasr_transcribe on the same features. */
int wasr_transcribe_device(WasrModel* m, const float* feats, const int64_t* n_frames,
                           const float* sil, int n_utt, int prev, int blk, int post, uint32_t* ids,
                           int64_t* ids_off, int64_t ids_cap);

/* Host fbank (src/fbank.rs:79-161): int16 PCM -> CMS-normalised [frames][40] fp32 and the
 * utterance's silence frame.  Returns the frame count (or, if feats is NULL, the count only). */
int64_t wasr_fbank(const int16_t* pcm, int64_t n, float* feats, int64_t cap, float* sil);

/* The same fbank on the GPU, batched over n utterances (src/fbank.rs:79-156; no counterpart
 * in the reference's C ABI, where fbank always runs in the Rust shell).  All pointers are
 * device pointers on the current device:
 *   pcm   int16 samples of all utterances, utterance i at [soff[i], soff[i+1]);
 *   soff  [n+1] sample offsets;  foff [n+1] frame offsets, foff[i+1] - foff[i] =
 *         (soff[i+1] - soff[i] - 400) / 160 + 1, or 0 below 400 samples;
 *   raw   scratch, frames x 40 doubles;  feats frames x 40 floats;  sil n x 40 floats (each
 *         utterance's CMS-normalised silence frame).
 * Stream-ordered on `stream`; returns 0, -1 for a null pointer, -4 for a launch failure.
 * The f32 features equal wasr_fbank's except where CUDA's double log and the host libm's differ
 * in the last place and the result sits on an f32 rounding boundary. */
int wasr_fbank_device(const int16_t* pcm, const int64_t* soff, const int64_t* foff, int n, int64_t frames,
                      double* raw, float* feats, float* sil, void* stream);

/* Streaming fbank (src/fbank.rs:122-161, the reference's Fbank): PCM arrives in pieces.
 *   wasr_fbank_stream_pending: frames a push of n more samples would emit.
 *   wasr_fbank_stream_push: appends n samples and writes the frames they complete to feats
 *     ([frames][40] host fp32, cap frames); returns the frame count, or -1 (nothing consumed)
 *     when cap is short.  Each frame is normalised by the 50-frame rolling mean as it stands
 *     after that frame, so the frames of any split equal wasr_fbank's frames of the whole.
 *   wasr_fbank_stream_silence: the silence frame under the rolling mean as it stands now
 *     (Fbank::silence, which the stream schedule pads its windows with). */
typedef struct WasrFbank WasrFbank;
WasrFbank* wasr_fbank_stream_create(void);
void wasr_fbank_stream_destroy(WasrFbank* st);
int64_t wasr_fbank_stream_pending(const WasrFbank* st, int64_t n);
int64_t wasr_fbank_stream_push(WasrFbank* st, const int16_t* pcm, int64_t n, float* feats, int64_t cap);
int wasr_fbank_stream_silence(const WasrFbank* st, float* sil);

/* CTC collapse (Model::text without the vocabulary, src/model.rs:622-642): drop repeats
 * and blank id 0.  Returns the collapsed length. */
int64_t wasr_ctc_collapse(const uint32_t* ids, int64_t n, uint32_t* out);

/* Parity hook: evaluates the kernels' restatements of the libm functions the reference CPU
 * path calls (fn 0: tanhf, 1: expf, 2: GELU of src/model.rs:710-712, 3: expm1f; 4: tanhf and
 * 5: GELU in the packed two-element form the GELU kernel runs; 6: the attention softmax's
 * division, y[2i] = x[2i] / x[2i+1] for numerators in [0, 1] and row sums in [1, 2^24)) on n
 * device floats, so tests can compare them bit for bit with the host's glibc / IEEE division. */
int wasr_eval_math(int fn, const float* x, float* y, int n, void* stream);

/* GELU + per-row int8 quantisation of a read-only device input y [m][k] (quant(gelu(f)) of
 * src/model.rs:495-496, src/kernels.rs:11-25, without writing the GELU values back; no
 * counterpart in the reference ABI, whose wk_gelu_quant works in place).  exact = 0 runs the
 * engine's kernel: for k = 2048 the certified one, which evaluates GELU with a cheap
 * approximation of bounded error, takes the row maximum from the exact GELU of the candidate
 * elements and quantises the elements whose scaled value lies within the error bound of a
 * rounding boundary again from the exact GELU -- the int8 row and scale are identical to the
 * exact computation's.  exact = 1 runs the all-exact kernel.  0, -1 for a null pointer, -2
 * for k too large, -4 for a launch failure. */
int wasr_gelu_quant(const float* y, int m, int k, int8_t* xq, float* xs, int exact, void* stream);

/* conv3 followed by the per-row int8 quantisation of its output (src/model.rs:446-468 and 489:
 * quant(y3, FLAT)) as the engine runs it, on device buffers: y2 [rows][64][41], c3 [192][576],
 * prep scratch of 576 * 192 + 192 floats (filled here), roff device row offsets of nseg windows
 * (NULL: one window of `rows`), xq [rows][3840] int8 and xs [rows].  No counterpart in the
 * reference ABI.  The products are summed with fused multiply-adds and bounded against the
 * reference's dotf order; the row maximum and every element whose scaled value lies within the
 * bound of a rounding boundary are evaluated in the reference's order, so xq and xs equal
 * quant(conv3(y2)) exactly.  0, -1 for bad arguments, -4 for a launch failure. */
int wasr_conv3_quant(const float* y2, const float* c3, float* prep, const int* roff, int nseg, int rows,
                     int8_t* xq, float* xs, void* stream);

/* conv1 of the conv frontend (src/model.rs:398-418) on device buffers: x [frames][40],
 * c1 [32][25], y1 [frames][32][40].  by_value = 1 runs the engine's kernel, which takes the
 * weights as a kernel argument (this call copies them to the host first and waits for the copy);
 * 0 the kernel of the reference ABI's wk_front.  foff: device frame prefix offsets of nseg
 * windows stacked in x, or NULL for one window.  Both keep the reference's dotf order, so y1
 * equals the CPU's bit for bit.  No counterpart in the reference ABI (a parity hook).  Returns 0,
 * -1 (arguments) or -4 (copy or launch). */
int wasr_conv1(const float* x, const float* c1, const int* foff, int nseg, int frames, int by_value, float* y1,
               void* stream);

/* conv2 of the conv frontend (src/model.rs:420-444) on device buffers: y1 [frames][32][40],
 * c2 [64][1568], y2 [rows][64][41] (column 40 written 0).  c2t: scratch of 64 * 1568 floats,
 * filled here with the transposed weights, selects the engine's position-pair kernel; NULL runs
 * the kernel of the reference ABI's wk_front (csrc/wtl_kern.cu:409-462).  foff / roff: device
 * frame / row prefix offsets of nseg windows stacked in y1 / y2, or both NULL for one window.
 * Both kernels keep the reference's dotf order, so y2 equals the CPU's bit for bit.  No
 * counterpart in the reference ABI (a parity hook).  Returns 0, -1 (arguments) or -4 (launch). */
int wasr_conv2(const float* y1, const float* c2, float* c2t, const int* foff, const int* roff, int nseg, int frames,
               int rows, float* y2, void* stream);

/* The engine's fused feed-forward up-projection (src/model.rs:495-496 with quant,
 * src/kernels.rs:11-25) on device buffers: q [M][N] int8 and qs [M] equal quant(gelu(x)) for
 * x = (acc * xs[row]) * ws[col] + bias[col] (ws_vec / bias may be NULL: ws, 0), acc the int32
 * products of a [M][K] and w [N][K]; the fp32 x is never stored.  work: M + 2 ints, work[0] the
 * error word (0 on entry; a bounded wait that gave up writes its code), the rest the list of rows
 * left to the exact kernel.  Shapes: K a multiple of 128 up to 2048, N a multiple of 256 up to
 * 2048, a / w / q 16-byte aligned.  No counterpart in the reference ABI (a parity hook).
 * Returns 0, -1 (arguments or shape) or -4 (launch). */
int wasr_gemm_gelu_quant(const int8_t* a, const float* xs, const int8_t* w, float ws, const float* ws_vec,
                         const float* bias, int M, int K, int N, int8_t* q, float* qs, int* work, void* stream);

/* Failure-handling probe of the same kernel (no counterpart in the reference ABI): its producer
 * issues no loads, so the bounded wait for the first operands runs out after wait_ns
 * (0 < wait_ns <= 1e9) with nothing in flight; the kernel writes a nonzero code to work[0] (0 on
 * entry), frees its tensor memory and returns, and the stream stays usable.  q and qs receive no
 * meaningful values.  Returns 0, -1 / -2 (arguments) or -4 (launch). */
int wasr_gemm_gelu_quant_wait_probe(const int8_t* a, const float* xs, const int8_t* w, float ws, const float* ws_vec,
                                    const float* bias, int M, int K, int N, int8_t* q, float* qs, int* work,
                                    unsigned long long wait_ns, void* stream);

/* Parity hook for the certified GELU: scans the float bit patterns [start, start + count)
 * (both even, start + count <= 2^32) and accumulates into the device array stats[8] (zeroed by
 * the caller), with g~ the approximation and g the exact GELU: [0] the largest |g~ - g| - B |g~|
 * over inputs where both are finite (the bits of a double), [1] inputs where g is non-finite and
 * g~ finite, [2] inputs where |g~ - g| > A + B |g~|, [3] inputs where only g~ is non-finite,
 * [4] the largest |g~ - g| / |g~| over |g~| >= 2^-20 and [5] the largest |g~ - g| below it
 * (double bits), [6] adjacent floats 0 <= x < x' <= inf with g(x') < g(x), [7] the largest
 * |g(x)| over non-NaN x < 0 (double bits).  0, or -1 for bad arguments. */
int wasr_gelu_cert_scan(unsigned long long start, unsigned long long count, unsigned long long* stats,
                        void* stream);

/* Measurement hook, no counterpart in the reference: the dense int8 tensor-core rate of this
 * GPU.  Launches `ctas` CTAs (one per SM) on `stream`; each issues iters x 4 back-to-back
 * tcgen05.mma kind::i8 of M = 128, N = 256, K = 32 from shared memory with no loads, i.e.
 * ctas * iters * 4 * 2 * 128 * 256 * 32 int8 ops; the caller times it with events.  *err (device
 * int, zeroed by the caller) receives a nonzero code if the completion wait ran out.  0, -1 for
 * bad arguments, -4 if the launch failed. */
int wasr_i8_mma_peak(int iters, int ctas, int* err, void* stream);

const char* wasr_version(void);

#ifdef __cplusplus
}
#endif
#endif /* WASR_H */
