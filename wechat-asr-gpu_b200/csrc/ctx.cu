// ctx.cu -- the reference's wp_* C ABI (csrc/wtlgpu.h) on top of the tcgen05 GEMM.
//
// Semantics mirrored from csrc/wtlgpu.cu: argument checks and return codes (:536-538,
// :715-748), the legacy-default-stream call stream that switches for good to a private
// capturable stream at the first capture (:751-775), capture end that always leaves the
// stream out of capture mode (:777-825), replay / graph free / node count (:827-847).
// What differs: no cuBLASLt handle, no algorithm search or disk cache, no padded weight
// copies (the GEMM handles any n), and a device error word that wp_sync reports.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/wtlgpu.h"
#include "gemm.cuh"
#include "kern.cuh"

using namespace wasr;

struct WpCtx {
  int dev = 0;
  cudaStream_t call_stream = nullptr;  // nullptr == legacy default stream
  cudaStream_t graph_stream = nullptr;
  int capturing = 0;
  size_t last_graph_nodes = 0;
  uint8_t* w = nullptr;
  size_t w_bytes = 0;
  float* scratch = nullptr;  // fp32 [t][n] staging of wp_gemm_q / wp_gemm_qg
  size_t scratch_bytes = 0;
  unsigned* rowmax = nullptr;
  size_t rowmax_n = 0;
  int* err_host = nullptr;  // mapped pinned error word
  int* err_dev = nullptr;
  std::mutex mu;
};

static bool stream_capturing(cudaStream_t s) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (s) cudaStreamIsCapturing(s, &cs);
  return cs != cudaStreamCaptureStatusNone;
}

// sized at create for t <= 512 rows of n <= 4096, so engine shapes never grow it in capture
static constexpr size_t kScratchInit = 512ull * 4096 * 4;
static constexpr size_t kRowmaxInit = 4096;

extern "C" {

const char* wp_version(void) {
  return "wasr-b200 wtlgpu 2.0 (tcgen05 kind::i8 sm_100a, TMA + TMEM; wp_gemm/2/q/qg; cuda-graph)";
}

WpCtx* wp_create(const void* w_host, size_t bytes) {
  WpCtx* c = new WpCtx();
  cudaGetDevice(&c->dev);
  gemm_prepare();
  kern_prepare();
  if (cudaStreamCreateWithFlags(&c->graph_stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete c;
    return nullptr;
  }
  c->call_stream = nullptr;
  if (cudaHostAlloc(reinterpret_cast<void**>(&c->err_host), sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->err_dev), c->err_host, 0) != cudaSuccess) {
    wp_destroy(c);
    return nullptr;
  }
  *c->err_host = 0;
  c->scratch_bytes = kScratchInit;
  c->rowmax_n = kRowmaxInit;
  if (cudaMalloc(&c->scratch, c->scratch_bytes) != cudaSuccess ||
      cudaMalloc(&c->rowmax, c->rowmax_n * sizeof(unsigned)) != cudaSuccess) {
    wp_destroy(c);
    return nullptr;
  }
  c->w_bytes = bytes;
  if (bytes > 0) {
    if (cudaMalloc(&c->w, bytes) != cudaSuccess) {
      wp_destroy(c);
      return nullptr;
    }
    if (w_host) {
      if (cudaMemcpy(c->w, w_host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        wp_destroy(c);
        return nullptr;
      }
    } else {
      cudaMemset(c->w, 0, bytes);
    }
  }
  return c;
}

void wp_destroy(WpCtx* c) {
  if (!c) return;
  cudaDeviceSynchronize();
  if (c->w) cudaFree(c->w);
  if (c->scratch) cudaFree(c->scratch);
  if (c->rowmax) cudaFree(c->rowmax);
  if (c->err_host) cudaFreeHost(c->err_host);
  if (c->graph_stream) cudaStreamDestroy(c->graph_stream);
  delete c;
}

void* wp_alloc(size_t bytes) {
  void* p = nullptr;
  if (bytes == 0) return nullptr;
  return cudaMalloc(&p, bytes) == cudaSuccess ? p : nullptr;
}
void wp_free(void* p) {
  if (p) cudaFree(p);
}

int wp_h2d(void* dev, const void* host, size_t bytes) {
  if (!dev || !host) return -1;
  return cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -2;
}
int wp_d2h(void* host, const void* dev, size_t bytes) {
  if (!host || !dev) return -1;
  return cudaMemcpy(host, dev, bytes, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -2;
}
void* wp_devptr(WpCtx* c, size_t off) {
  if (!c || off > c->w_bytes) return nullptr;
  return c->w + off;
}
int wp_sync(WpCtx* c) {
  if (!c) return -1;
  if (cudaStreamSynchronize(c->call_stream) != cudaSuccess) return -2;
  if (*reinterpret_cast<volatile int*>(c->err_host)) {
    *c->err_host = 0;
    return -21;
  }
  return 0;
}
int wp_set_stream(WpCtx* c, void* stream) {
  if (!c) return -1;
  if (c->capturing) return -16;
  c->call_stream = static_cast<cudaStream_t>(stream);
  return 0;
}
void* wp_stream(WpCtx* c) { return c ? static_cast<void*>(c->call_stream) : nullptr; }
size_t wp_scratch_bytes(WpCtx* c) { return c ? c->scratch_bytes : 0; }

}  // extern "C"

// One GEMM call of the wp_gemm family.  mode 0: fp32 out; 1: re-quant; 2: GELU + re-quant;
// 3: raw int32.  ws_vec (nullable) gives per-output-channel scales.
static int gemm_impl(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
                     const float* ws_vec, const float* bias, cudaStream_t stream, float* out, int8_t* out_q,
                     float* out_s, int32_t* out_i32, int mode) {
  if (!c || !xq || (mode != 3 && !xs)) return -1;
  if (mode == 3 ? !out_i32 : (out_q ? !out_s : !out)) return -1;
  if (t <= 0 || k <= 0 || n <= 0) return 0;
  if (static_cast<size_t>(n) * static_cast<size_t>(k) > c->w_bytes ||
      w_off > c->w_bytes - static_cast<size_t>(n) * static_cast<size_t>(k))
    return -2;
  std::lock_guard<std::mutex> lock(c->mu);
  GemmArgs g{};
  g.a = xq;
  g.b = reinterpret_cast<const int8_t*>(c->w + w_off);
  g.M = t;
  g.N = n;
  g.K = k;
  g.n_store = n;
  g.xs = xs;
  g.ws = ws;
  g.ws_vec = ws_vec;
  g.bias = bias;
  g.ldo = n;
  g.err = c->err_dev;
  if (mode == 0) {
    g.out = out;
    g.epi = EPI_F32;
    return gemm_run(g, stream);
  }
  if (mode == 3) {
    g.out_i32 = out_i32;
    g.epi = EPI_I32;
    return gemm_run(g, stream);
  }
  // re-quant modes: fp32 staging + per-row |max|, then quantise with that max
  const size_t need = static_cast<size_t>(t) * n * sizeof(float);
  if (need > c->scratch_bytes || static_cast<size_t>(t) > c->rowmax_n) {
    if (stream_capturing(stream)) return -5;
    cudaStreamSynchronize(stream);
    if (need > c->scratch_bytes) {
      float* ns = nullptr;
      if (cudaMalloc(&ns, need + need / 2) != cudaSuccess) return -5;
      cudaFree(c->scratch);
      c->scratch = ns;
      c->scratch_bytes = need + need / 2;
    }
    if (static_cast<size_t>(t) > c->rowmax_n) {
      unsigned* nr = nullptr;
      if (cudaMalloc(&nr, static_cast<size_t>(t) * 2 * sizeof(unsigned)) != cudaSuccess) return -5;
      cudaFree(c->rowmax);
      c->rowmax = nr;
      c->rowmax_n = static_cast<size_t>(t) * 2;
    }
  }
  if (cudaMemsetAsync(c->rowmax, 0, static_cast<size_t>(t) * sizeof(unsigned), stream) != cudaSuccess) return -4;
  g.out = c->scratch;
  g.rowmax = c->rowmax;
  g.epi = mode == 2 ? EPI_GELU_ROWMAX : EPI_F32_ROWMAX;
  int rc = gemm_run(g, stream);
  if (rc) return rc;
  return launch_quant_rows_max(c->scratch, t, n, c->rowmax, out_q, out_s, stream);
}

extern "C" {

int wp_gemm(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
            size_t bias_off, float* out) {
  const float* bias = nullptr;
  if (c && bias_off != static_cast<size_t>(-1)) {
    if (bias_off + static_cast<size_t>(n) * 4 > c->w_bytes) return -2;
    bias = reinterpret_cast<const float*>(c->w + bias_off);
  }
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias, c ? c->call_stream : nullptr, out, nullptr, nullptr,
                   nullptr, 0);
}

int wp_gemm2(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
             const float* bias_dev, void* stream, float* out) {
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias_dev, static_cast<cudaStream_t>(stream), out, nullptr,
                   nullptr, nullptr, 0);
}

int wp_gemm_q(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
              const float* bias_dev, void* stream, int8_t* out_q, float* out_s) {
  if (!out_q) return -1;
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias_dev, static_cast<cudaStream_t>(stream), nullptr,
                   out_q, out_s, nullptr, 1);
}

int wp_gemm_qg(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
               const float* bias_dev, void* stream, int8_t* out_q, float* out_s) {
  if (!out_q) return -1;
  return gemm_impl(c, xq, xs, t, k, w_off, n, ws, nullptr, bias_dev, static_cast<cudaStream_t>(stream), nullptr,
                   out_q, out_s, nullptr, 2);
}

int wp_gemm2_pc(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, const float* ws_dev,
                const float* bias_dev, void* stream, float* out) {
  if (!ws_dev) return -1;
  return gemm_impl(c, xq, xs, t, k, w_off, n, 0.0f, ws_dev, bias_dev, static_cast<cudaStream_t>(stream), out,
                   nullptr, nullptr, nullptr, 0);
}

int wp_gemm_i32(WpCtx* c, const int8_t* xq, int t, int k, size_t w_off, int n, void* stream, int32_t* acc) {
  return gemm_impl(c, xq, nullptr, t, k, w_off, n, 0.0f, nullptr, nullptr, static_cast<cudaStream_t>(stream),
                   nullptr, nullptr, nullptr, acc, 3);
}

}  // extern "C"

// ------------------------------------------------------------------------ no-allocation GEMM+quant
// Some callers cannot call cudaMalloc at the time they run a GEMM: code running while a CUDA
// graph is being captured (an allocation is not a capturable operation), or an embedding
// process whose memory budget is fixed up front.  wp_gemm_q grows its fp32 staging buffer on
// demand; wp_gemm_q_noalloc instead stages through this fixed array, which every GPU that loads
// the library holds until the process exits: WP_NOALLOC_MAX_ELEMS fp32 values of GEMM output
// (t*n <= 1,048,576, 4 MiB) followed by WP_NOALLOC_MAX_ROWS per-row maxima (t <= 4096).
static __device__ __align__(256) float g_noalloc_scratch[WP_NOALLOC_MAX_ELEMS + WP_NOALLOC_MAX_ROWS];

// Device address of g_noalloc_scratch per device.  In host code the array's name is only a
// host-side stand-in, so the address is looked up with cudaGetSymbolAddress once per device,
// with that device current.
static std::mutex g_noalloc_mu;
static float* g_noalloc_addr[64] = {};

static int noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -23;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "[wasr] wp_gemm_q_noalloc: cudaGetSymbolAddress failed: %s\n", cudaGetErrorString(e));
      cudaGetLastError();
      return -23;
    }
    g_noalloc_addr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_addr[dev];
  return 0;
}

extern "C" {

int wp_gemm_q_noalloc(WpCtx* c, const int8_t* xq, const float* xs, int t, int k, size_t w_off, int n, float ws,
                      const float* bias_dev, void* stream, int8_t* out_q, float* out_s) {
  if (!c || !xq || !xs || !out_q || !out_s) return -1;
  if (t <= 0 || k <= 0 || n <= 0) return 0;
  if (static_cast<size_t>(n) * static_cast<size_t>(k) > c->w_bytes ||
      w_off > c->w_bytes - static_cast<size_t>(n) * static_cast<size_t>(k))
    return -2;
  if (t > WP_NOALLOC_MAX_ROWS || static_cast<size_t>(t) * static_cast<size_t>(n) > WP_NOALLOC_MAX_ELEMS) {
    fprintf(stderr,
            "[wasr] wp_gemm_q_noalloc: t=%d, n=%d exceeds the static scratch (t <= %d, t*n <= %d); "
            "use wp_gemm_q\n",
            t, n, WP_NOALLOC_MAX_ROWS, WP_NOALLOC_MAX_ELEMS);
    return -22;
  }
  float* scratch = nullptr;
  if (const int rc = noalloc_scratch(&scratch)) return rc;
  unsigned* rowmax = reinterpret_cast<unsigned*>(scratch + WP_NOALLOC_MAX_ELEMS);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::lock_guard<std::mutex> lock(c->mu);
  // the array keeps the previous call's values: the row maxima must start from zero
  if (cudaMemsetAsync(rowmax, 0, static_cast<size_t>(t) * sizeof(unsigned), st) != cudaSuccess) return -4;
  GemmArgs g{};
  g.a = xq;
  g.b = reinterpret_cast<const int8_t*>(c->w + w_off);
  g.M = t;
  g.N = n;
  g.K = k;
  g.n_store = n;
  g.xs = xs;
  g.ws = ws;
  g.bias = bias_dev;
  g.ldo = n;
  g.err = c->err_dev;
  g.out = scratch;
  g.rowmax = rowmax;
  g.epi = EPI_F32_ROWMAX;
  const int rc = gemm_run(g, st);
  if (rc) return rc;
  return launch_quant_rows_max(scratch, t, n, rowmax, out_q, out_s, st);
}

int wp_quant_rows(const float* y, int t, int n, void* stream, int8_t* out_q, float* out_s) {
  if (!y || !out_q || !out_s) return -1;
  if (t <= 0 || n <= 0) return 0;
  if (n > 65536) return -7;
  return launch_quant_rows(y, t, n, n, out_q, out_s, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------ CUDA graphs
int wp_capture_begin(WpCtx* c) {
  if (!c) return -1;
  if (c->capturing) {
    fprintf(stderr, "[wasr] capture already in progress\n");
    return -10;
  }
  if (!c->graph_stream) return -10;
  if (c->call_stream == nullptr) {
    // the legacy stream cannot be captured: drain it, then move to the private stream for good
    cudaError_t se = cudaStreamSynchronize(nullptr);
    if (se != cudaSuccess) {
      cudaGetLastError();
      return -10;
    }
    c->call_stream = c->graph_stream;
  }
  if (cudaStreamBeginCapture(c->call_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return -10;
  }
  c->capturing = 1;
  return 0;
}

int wp_capture_end(WpCtx* c, void** out_exec) {
  if (!c || !out_exec) return -1;
  *out_exec = nullptr;
  if (!c->capturing) return -12;
  cudaStream_t s = c->call_stream;
  c->capturing = 0;
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(s, &g);
  if (e != cudaSuccess) {
    cudaGetLastError();
    if (stream_capturing(s)) {
      cudaGraph_t g2 = nullptr;
      cudaStreamEndCapture(s, &g2);
      if (g2) cudaGraphDestroy(g2);
      cudaGetLastError();
    }
    return -13;
  }
  if (!g) return -14;
  size_t nodes = 0;
  cudaGraphGetNodes(g, nullptr, &nodes);
  c->last_graph_nodes = nodes;
  if (nodes == 0) {
    cudaGraphDestroy(g);
    return -14;
  }
  cudaGraphExec_t ex = nullptr;
  e = cudaGraphInstantiate(&ex, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return -15;
  }
  *out_exec = ex;
  return 0;
}

int wp_replay(WpCtx* c, void* exec) {
  if (!c || !exec) return -1;
  if (cudaGraphLaunch(static_cast<cudaGraphExec_t>(exec), c->call_stream) != cudaSuccess) {
    cudaGetLastError();
    return -17;
  }
  return 0;
}

int wp_graph_free(WpCtx* c, void* exec) {
  (void)c;
  if (!exec) return 0;
  if (cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(exec)) != cudaSuccess) {
    cudaGetLastError();
    return -18;
  }
  return 0;
}

size_t wp_graph_count(WpCtx* c) { return c ? c->last_graph_nodes : 0; }
int wp_is_capturing(WpCtx* c) { return c ? c->capturing : 0; }

}  // extern "C"
