/* wasr_oracle.h -- CPU restatement of the reference's CPU path (TEST INFRASTRUCTURE).
 *
 * This is the parity oracle and the timed CPU baseline.  It is never linked into, loaded by
 * or called from the product (libwasr_gpu.so); only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / `--impl reference` leg use it, and only as the checker.
 *
 * The reference CPU path is Rust (src/kernels.rs, src/model.rs, src/fbank.rs,
 * src/stream.rs); no Rust toolchain exists here, so each function below restates one Rust
 * function in C with the same floating-point operation order (no FMA contraction:
 * compiled with -ffp-contract=off, as rustc never contracts).  Pinning: the only
 * known-answer test the reference ships is src/kernels.rs:185-208 (qgemm vs a scalar dot
 * product on an LCG input); tests/test_oracle.py reproduces it, and cross-checks the int32
 * accumulators against an independent numpy int64 matmul.  The reference ships no golden
 * outputs, weights or audio (they are gitignored there), so model-level parity is pinned
 * only through this restatement.
 */
#ifndef WASR_ORACLE_H
#define WASR_ORACLE_H

#include <stdint.h>

#include "../include/wasr.h"

#ifdef __cplusplus
extern "C" {
#endif

void wo_set_threads(int n);
int wo_get_threads(void);

/* src/kernels.rs:11-25 */
void wo_quant(const float* x, int64_t t, int k, int8_t* q, float* s);
/* src/kernels.rs:87-97 (scalar dot1, exact int32) */
int32_t wo_dot1(const int8_t* a, const int8_t* b, int k);
/* src/kernels.rs:33-63 with the x86 AVX2 dot2x4 of src/kernels.rs:131-168 when k % 32 == 0.
 * ws_vec (nullable) generalises the per-tensor scale to per output channel. */
void wo_qgemm(const int8_t* xq, const float* xs, int64_t t, int k, const int8_t* w, int n, float ws,
              const float* ws_vec, const float* bias, float* out);
/* exact int32 accumulators via the scalar dot1 */
void wo_qgemm_acc(const int8_t* xq, int64_t t, int k, const int8_t* w, int n, int32_t* acc);
/* src/kernels.rs:172-183 */
float wo_dotf(const float* a, const float* b, int n);
/* src/model.rs:693-704 */
void wo_norm(const float* x, int64_t t, int d, const float* g, const float* b, float* y);
/* src/model.rs:710-712 */
float wo_gelu(float x);
/* the host libm (glibc) functions the reference calls, over arrays (parity checks) */
void wo_libm_tanhf(const float* x, float* y, int64_t n);
void wo_libm_expf(const float* x, float* y, int64_t n);
void wo_gelu_array(const float* x, float* y, int64_t n);
/* src/model.rs:714-739: q,k,v,out are [t][512] */
void wo_attention(const float* q, const float* k, const float* v, int t, float* out);
/* src/model.rs:389-478: x [t][40] -> y3 [t1][3840]; returns t1 (0 if t < 5) */
int wo_frontend(const float* x, int t, const float* c1, const float* c2, const float* c3, float* y3);
/* the conv1 stage alone (src/model.rs:398-418): x [t][40] -> y1 [t][32][40] */
void wo_conv1(const float* x, int t, const float* c1, float* y1);
/* the conv2 stage alone (src/model.rs:420-444): y1 [t][32][40] -> y2 [t1][64][41] */
void wo_conv2(const float* y1, int t, const float* c2, float* y2);
/* the conv3 stage alone (src/model.rs:446-468): y2 [t1][64][41] -> y3 [t1][3840] */
void wo_conv3(const float* y2, int t1, const float* c3, float* y3);
/* src/model.rs:368-386,480-502: whole forward of one window; ids [t1]; logits (nullable)
 * [t1][vocab]; returns t1 */
int wo_forward(const uint8_t* blob, const WasrPlan* plan, const float* x, int t, uint32_t* ids,
               float* logits);
/* src/model.rs:488-502 from y3 (after the frontend); returns t1 */
int wo_run_post(const uint8_t* blob, const WasrPlan* plan, int t1, const float* y3, uint32_t* ids,
                float* logits);
/* src/model.rs:499-500 */
uint32_t wo_argmax(const float* row, int n);
/* src/model.rs:622-642 without the vocabulary: drop repeats, drop blank 0 */
int64_t wo_ctc(const uint32_t* ids, int64_t n, uint32_t* out);
/* src/fbank.rs:79-102: one frame of 400 samples -> 40 f64 values */
void wo_fbank_frame(const int16_t* x, double* out);
/* src/fbank.rs:128-161 (whole utterance pushed at once): returns frame count; feats may be
 * NULL to count; sil receives Fbank::silence() after the last frame. */
int64_t wo_fbank(const int16_t* pcm, int64_t n, float* feats, int64_t cap, float* sil);
/* src/stream.rs:58-70,128-147,159-168 in batch mode: the whole utterance is pushed, then
 * finish().  ids receives the per-frame ids before CTC collapse; returns their count, or -1
 * if ids_cap is too small.  n_fwd (nullable) receives the number of forward calls. */
int64_t wo_transcribe(const uint8_t* blob, const WasrPlan* plan, const float* feats, int64_t n,
                      const float* sil, int prev, int blk, int post, uint32_t* ids, int64_t ids_cap,
                      int* n_fwd);
/* src/stream.rs:128-168 for features arriving in pieces: push's commit loop, and the ids of
 * partial() (finish = 0) or finish() (finish = 1). */
int wo_stream_commit(const uint8_t* blob, const WasrPlan* plan, const float* feats, int64_t n,
                     const float* sil, int prev, int blk, int post, int64_t* s, uint32_t* ids,
                     int64_t* n_ids, int64_t cap, int* n_fwd);
int64_t wo_stream_tail(const uint8_t* blob, const WasrPlan* plan, const float* feats, int64_t n,
                       const float* sil, int prev, int64_t s, const uint32_t* ids, int64_t n_ids,
                       int finish, uint32_t* out, int64_t cap, int* n_fwd);
/* Model::text (src/model.rs:620-642) and tidy (src/stream.rs:203-210), UTF-8 */
int64_t wo_text(const uint32_t* ids, int64_t n, const char* const* vocab, int64_t n_vocab, char* out, int64_t cap);
int64_t wo_tidy(char* s, int trim_end);

#ifdef __cplusplus
}
#endif
#endif
