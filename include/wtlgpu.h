/* wtlgpu.h -- the reference-facing C ABI of libwasr_gpu.so, rebuilt for B200 (sm_100a).
 *
 * Every declaration below is an entry point the reference's Rust shell binds
 * (src/gpu.rs:13-86) or that the reference library exports (csrc/wtlgpu.h:35-105,
 * csrc/wtl_kern.cu:409-462, csrc/wk_attention_*.cu, csrc/wk_attn_api.cu).  Names,
 * argument order, argument meaning, return codes and stream behaviour are kept so that
 * `wasr --gpu` links against this library unchanged.  The implementation behind them is
 * new: a tcgen05 int8 GEMM (TMA-fed, TMEM accumulators) replaces cuBLASLt, and hand-written
 * sm_100a kernels replace the SIMT/cuBLAS attention and small ops.
 *
 * Layout contract (row-major throughout, as in the reference CPU path src/kernels.rs):
 *   w    : [n][k] int8 at byte offset w_off inside the weight blob
 *   xq   : [t][k] int8, xs : [t] fp32 per-row activation scale
 *   out  : [t][n] fp32,  out[i][j] = ((float)acc[i][j] * xs[i]) * ws + bias[j]
 * The epilogue multiplies in the CPU path's order (src/kernels.rs:53), so outputs are
 * bit-identical to it (the reference GPU library used acc * (xs*ws) instead).
 *
 * Streams: every call runs on the context's call stream (wp_stream), which is the legacy
 * default stream until the first wp_capture_begin and the context's private capturable
 * stream afterwards (csrc/wtlgpu.cu:751-775).  Callers re-query wp_stream before each
 * launch of their own, exactly as src/gpu.rs:170-173 does.
 *
 * Shape warm-up: nothing in this library searches for algorithms or grows buffers lazily
 * on a hot call except the fp32 scratch of wp_gemm_q / wp_gemm_qg, which is sized at
 * wp_create for t <= 512 rows of n <= 16384.  Calls inside a capture therefore never
 * return -5 / -6 for the shapes the engine uses; larger shapes outside a capture grow the
 * scratch, and inside a capture return -5 like the reference.
 *
 * Error codes (csrc/wtlgpu.h:80-95, csrc/wtlgpu.cu:536-846): -1 bad argument, -2 offset
 * out of the blob, -4 kernel launch failed, -5 scratch too small during capture,
 * -7 unsupported quant shape, -10 capture begin, -12 end without begin, -13 capture
 * invalidated, -14 empty graph, -15 instantiate failed, -16 set_stream while capturing,
 * -17 replay failed, -18 graph free failed, -21 a bounded device wait gave up.
 */
#ifndef WTLGPU_H
#define WTLGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct WpCtx WpCtx;

/* ---- context, memory, copies ------------------------------------------------------ */
/* Replaces wp_create (csrc/wtlgpu.cu:635-659; bound at src/gpu.rs:15): copies the whole
 * weight blob to the current device once. */
WpCtx* wp_create(const void* w_host, size_t bytes);
/* Replaces wp_destroy (csrc/wtlgpu.cu:661-680; src/gpu.rs:16). */
void wp_destroy(WpCtx* c);
/* Replace wp_alloc / wp_free (csrc/wtlgpu.cu:682-687; src/gpu.rs:17-18). */
void* wp_alloc(size_t bytes);
void wp_free(void* p);
/* Replace wp_h2d / wp_d2h (csrc/wtlgpu.cu:689-696; src/gpu.rs:19-20): synchronous copies. */
int wp_h2d(void* dev, const void* host, size_t bytes);
int wp_d2h(void* host, const void* dev, size_t bytes);
/* Replaces wp_devptr (csrc/wtlgpu.cu:697-700; src/gpu.rs:21). */
void* wp_devptr(WpCtx* c, size_t off);
/* Replaces wp_sync (csrc/wtlgpu.cu:701-705; src/gpu.rs:22).  Also reports -21 if a kernel
 * of this context hit its bounded-wait limit since the last sync. */
int wp_sync(WpCtx* c);
/* Replace wp_set_stream / wp_stream / wp_scratch_bytes / wp_version
 * (csrc/wtlgpu.cu:706-713,631-633; wp_stream bound at src/gpu.rs:35). */
int wp_set_stream(WpCtx* c, void* stream);
void* wp_stream(WpCtx* c);
size_t wp_scratch_bytes(WpCtx* c);
const char* wp_version(void);

/* ---- int8 GEMM ------------------------------------------------------------------- */
/* Replaces wp_gemm (csrc/wtlgpu.cu:715-723; src/gpu.rs:23-34):
 * out[t][n] = (xq . w^T) * xs * ws + bias, bias given as a blob offset ((size_t)-1 = none). */
int wp_gemm(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n,
            float ws, size_t bias_off, float* out);
/* Replaces wp_gemm2 (csrc/wtlgpu.cu:725-728): device bias pointer and explicit stream. */
int wp_gemm2(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n,
             float ws, const float* bias_dev, void* stream, float* out);
/* Replaces wp_gemm_q (csrc/wtlgpu.cu:730-734): GEMM + bias, then per-row dynamic int8
 * re-quantisation of the result (src/kernels.rs:11-25 rounding). */
int wp_gemm_q(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n,
              float ws, const float* bias_dev, void* stream, int8_t* out_q, float* out_s);
/* Replaces wp_gemm_qg (csrc/wtlgpu.cu:736-740): GEMM + bias + GELU + per-row re-quant. */
int wp_gemm_qg(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n,
               float ws, const float* bias_dev, void* stream, int8_t* out_q, float* out_s);
/* Replaces wp_quant_rows (csrc/wtlgpu.cu:742-748).  The reference needs n % 256 == 0 and
 * n <= 4096 (-7 otherwise); this build accepts any n > 0 and keeps -7 only for n > 65536. */
int wp_quant_rows(const float* y, int t, int n, void* stream, int8_t* out_q, float* out_s);

/* ---- CUDA graphs (csrc/wtlgpu.cu:751-847; bound at src/gpu.rs:36-40) -------------- */
int wp_capture_begin(WpCtx* c);
int wp_capture_end(WpCtx* c, void** out_exec);
int wp_replay(WpCtx* c, void* exec);
int wp_graph_free(WpCtx* c, void* exec);
size_t wp_graph_count(WpCtx* c);
int wp_is_capturing(WpCtx* c);

/* ---- fused small ops (csrc/wtl_kern.cu:409-462; bound at src/gpu.rs:56-86) --------- */
/* conv frontend x[t][40] -> y1[t][32][40] -> y2[t1][64][41] -> y3[t1][3840]
 * (csrc/wtl_kern.cu:414-423; CPU semantics src/model.rs:389-478). */
void wk_front(void* stream, const float* x, const float* c1, const float* c2, const float* c3,
              int t, int t1, float* y1, float* y2, float* y3);
/* LayerNorm(h; g, b) -> per-row int8 (csrc/wtl_kern.cu:435-438; src/model.rs:693-704). */
void wk_norm_quant(void* stream, const float* h, const float* g, const float* b, int t, int d,
                   int8_t* xq, float* xs);
/* h += o, then LayerNorm -> int8 (csrc/wtl_kern.cu:440-443). */
void wk_add_norm_quant(void* stream, float* h, const float* o, const float* g, const float* b,
                       int t, int d, int8_t* xq, float* xs);
/* per-row int8 quant (csrc/wtl_kern.cu:445-447; src/kernels.rs:11-25). */
void wk_quant(void* stream, const float* x, int t, int k, int8_t* xq, float* xs);
/* in-place tanh-GELU then per-row quant (csrc/wtl_kern.cu:449-451; src/model.rs:710-712). */
void wk_gelu_quant(void* stream, float* x, int t, int k, int8_t* xq, float* xs);
/* h += a (csrc/wtl_kern.cu:453-456). */
void wk_add(void* stream, float* h, const float* a, int t, int d);
/* row argmax, first maximum wins (csrc/wtl_kern.cu:458-460; src/model.rs:499-500). */
void wk_argmax(void* stream, const float* x, int t, int n, uint32_t* out);
const char* wk_version(void);
int wk_last_error(void);

/* ---- attention (8 heads x 64, fp32): out[i][h*64+l] = sum_j softmax_j(q_i.k_j*0.125) v_j -- */
/* Replaces wk_attention_fast (csrc/wk_attn_api.cu:345-350; src/gpu.rs:44-54).  scratch is
 * accepted and ignored (the fused kernel keeps scores on chip). */
int wk_attention_fast(void* stream, const float* q, const float* k, const float* v, int t, int d,
                      int heads, float* scratch, float* out);
/* Replaces wk_attention (csrc/wtl_kern.cu:426-433; void in the reference). */
void wk_attention(void* stream, const float* q, const float* k, const float* v, int t, int d,
                  int heads, float* scratch, float* out);
/* Replace wk_attention_tiled / _tuned / _version (csrc/wk_attention_fast.cu:286-322). */
int wk_attention_tiled(void* stream, const float* q, const float* k, const float* v, int t, int d,
                       int heads, float* scratch, float* out);
int wk_attention_tiled_tuned(void* stream, const float* q, const float* k, const float* v, int t,
                             int d, int heads, float* out, int it, int ch);
const char* wk_attention_tiled_version(void);
/* Replace wk_attention_cublas / _part (csrc/wk_attention_cublas.cu:78-138).  No cuBLAS is
 * used: the name is kept for ABI completeness and runs the same fused kernel; _part 0/1
 * are no-ops and part 2 runs the whole attention. */
int wk_attention_cublas(void* stream, const float* q, const float* k, const float* v, int t, int d,
                        int heads, float* scratch, float* out);
int wk_attention_cublas_part(int part, void* stream, const float* q, const float* k,
                             const float* v, int t, int d, int heads, float* scratch, float* out);
/* Replaces wk_attention_version (csrc/wk_attn_api.cu:352-354). */
const char* wk_attention_version(void);

/* ---- additive: per-output-channel weight scales and raw accumulators -------------- */
/* wp_gemm2 with an fp32 [n] per-output-channel scale vector in device memory
 * (ws_dev != NULL replaces ws):  out = ((float)acc * xs[i]) * ws_dev[j] + bias[j]. */
int wp_gemm2_pc(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n,
                const float* ws_dev, const float* bias_dev, void* stream, float* out);
/* Raw int32 accumulators acc[t][n] = sum_k xq[i][k] * w[j][k] (parity hook). */
int wp_gemm_i32(WpCtx* c, const int8_t* xq, int t, int k, size_t w_off, int n, void* stream,
                int32_t* acc);

/* ---- additive: failure-handling test hook ---------------------------------------- */
/* No counterpart in the reference (its kernels have no bounded waits).  Every mbarrier wait in
 * the tcgen05 GEMM gives up after a limit (2 s by default), records the cause in the context's
 * error word and lets the kernel release its tensor memory and return; the next wp_sync then
 * returns -21.  This entry point runs one int32 GEMM (as wp_gemm_i32) whose producer issues no
 * loads, with every wait limited to wait_ns (1 ns .. 1 s), so that the waits run out with
 * nothing in flight.  The output is not written meaningfully.  -2 for a wait_ns outside that
 * range or k % 16 != 0 (the shapes without tensor-core waits). */
int wp_gemm_i32_wait_probe(WpCtx* c, const int8_t* xq, int t, int k, size_t w_off, int n, void* stream,
                           int32_t* acc, unsigned long long wait_ns);

/* ---- additive: GEMM + per-row re-quantisation that allocates nothing ------------- */
/* No counterpart in the reference.  Same result as wp_gemm_q, for callers that cannot
 * allocate device memory when they run it: a process whose framework has already handed the
 * GPU's memory to its own caching allocator (a cudaMalloc outside that pool fails), or a
 * latency-bound thread, such as the audio callback of a streaming recogniser, that must not
 * block in cudaMalloc / cudaFree (both can synchronise the device).  wp_gemm_q may cudaMalloc a
 * larger staging buffer on demand; this entry point stages through one fixed device array
 * inside the library instead, which every GPU that loads the library holds until the process
 * exits (4 MiB + 16 KiB).  Limits: t <= WP_NOALLOC_MAX_ROWS and t*n <= WP_NOALLOC_MAX_ELEMS;
 * larger calls return -22 and change nothing.  It runs on the context's device.  The first call
 * on each device looks up the array's device address (cudaGetSymbolAddress; -23 if that
 * fails); make that first call before any stream capture.  All calls share the one array,
 * which keeps the last call's values (every call clears the per-row maxima it uses).  Calls
 * that overlap on the GPU (on different streams or contexts) therefore race; serialise them. */
#define WP_NOALLOC_MAX_ELEMS 1048576
#define WP_NOALLOC_MAX_ROWS 4096
int wp_gemm_q_noalloc(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n,
                      float ws, const float* bias_dev, void* stream, int8_t* out_q, float* out_s);

#ifdef __cplusplus
}
#endif
#endif /* WTLGPU_H */
